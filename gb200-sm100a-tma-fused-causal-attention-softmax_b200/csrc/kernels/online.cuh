// Pipelined online-softmax causal kernel for long rows (the `online` kernel
// choice, and the automatic choice once a row pair no longer fits two stages
// of the row-resident kernel).
//
// Replaces gpu/src/main.rs:546-727 (two dense TMA passes, 2 KB tiles, one
// tile in flight per buffer, wait_group(0) after every store):
//
//  * each CTA owns whole rows (flat row index blockIdx.x + j*gridDim.x,
//    walked with a division-free cursor) and a ring of S shared-memory
//    tiles; a tile is W consumer warps x 32 lanes x
//    VPT 16-byte vectors (4 warps x 2 = 4 KB for rows of up to two default
//    tiles, 8 warps x 2 = 8 KB by default, 31 warps x 1 = 15.5 KB for rows
//    longer than the default ring, on the deepest ring that fits);
//  * one producer warp keeps the ring full with 1-D TMA bulk copies of the
//    causal prefix only, running ahead across row boundaries, and writes the
//    masked columns and pitch padding with bulk stores from a zero buffer;
//    it refills a stage once all W consumer warps have arrived on the
//    stage's `empty` mbarrier, so no CTA-wide barrier runs per tile;
//  * pass 1 keeps a per-lane online (max, sum) pair: the max of a vector is
//    taken on packed halves, the sum is rescaled only when that max grows,
//    and the exponents (x - m) * sl run on packed f32 pairs (x == m gives
//    exactly 0 at any scale, up to 1e30); the row's pairs are merged with a
//    redux max and a rescaled warp sum, and one consumer-only barrier per row;
//  * pass 2 writes p = 2^((x - M) * sl - log2 S), the reciprocal of the sum
//    folded into the exponent (one packed fma), as 16-byte vectors straight
//    from registers; a zero scale keeps 1 * RN(1/S). When the row fits the ring it
//    stays resident in shared memory between the passes, so HBM sees a single
//    read, and pass 2 hands each tile back as soon as it is written out, so
//    the next row's tiles stream in while this row's go out; longer rows are
//    fetched again for pass 2 (the first fetch leaves them in L2 with a
//    normal priority, the second marks them evict-first);
//  * a zero scale (every causal probability 1/valid) is a separate
//    instantiation of the consumer passes, so no per-element test of it runs.
//
// All mbarrier waits are bounded (Geometry::timeout_ns) and report
// kStatusTimeout through the status word; the consumers leave a row together
// (a barrier that ORs their verdicts), and the producer stops at the abort
// flag and waits, bounded, for its copies in flight before it returns.
#pragma once

#include "common.cuh"
#include "geometry.cuh"

namespace cs {

// Launch shapes: consumer warps and 16-byte vectors per lane and tile; one
// more warp is the producer.
constexpr int kOnlineConsumerWarps = 8;  // the default shape: 8 KB tiles
constexpr int kOnlineVecPerThread = 2;
constexpr int kOnlineThreads = 32 * (kOnlineConsumerWarps + 1);
constexpr int kOnlineTileVec = 32 * kOnlineConsumerWarps * kOnlineVecPerThread;  // 512 vectors
constexpr int kOnlineWideThreads = 1024;  // long rows: 31 consumer warps, one vector per lane
// Rows of at most two default tiles: 4 consumer warps (4 KB tiles), so that
// six CTAs, each with a ring of 8 stages, share an SM.
constexpr int kOnlineShortConsumerWarps = 4;
constexpr int kOnlineShortThreads = 32 * (kOnlineShortConsumerWarps + 1);
constexpr int kOnlineZeroBytes = 4096;    // zero buffer for the masked columns' bulk stores

// Vectors of one tile for a CTA of `threads` threads and VPT vectors per lane.
__host__ __device__ constexpr int online_tile_vec(int threads, int vpt) { return (threads - 32) * vpt; }

struct OnlineParams {
  Geometry g;
  int64_t total_rows;  // batch * rows
  int32_t stages;      // ring depth (tiles)
};

// Shared memory after the tiles: zero buffer, two rows' warp partials,
// full and empty mbarriers per stage, the abort flag.
__host__ __device__ constexpr int online_tail_bytes(int stages) {
  return kOnlineZeroBytes + 2 * 32 * 8 + 2 * stages * 8 + 16;
}

// The W consumer warps: both passes over every row of the CTA. A lane takes
// vectors warp*32 + lane + q*32W (q < VPT) of each tile, so each warp reads
// 512 contiguous bytes per load.
template <int VPT, bool kZeroScale>
__device__ __forceinline__ void online_consumers(const OnlineParams& p, const uint8_t* tiles, float2* red,
                                                 uint64_t* full, uint64_t* empty, volatile int* abort_flag,
                                                 int warp, int lane, int W) {
  const Geometry& g = p.g;
  const int S = p.stages;
  const int32_t tile_vec = 32 * W * VPT;
  const size_t tile_bytes = (size_t)tile_vec * 16;
  const float sl = g.scale * kLog2e;  // exponents (x - max) * scale*log2(e)
  const float2 sl2 = make_float2(sl, sl);
  const int32_t lv0 = warp * 32 + lane;
  RowCursor rows(g, blockIdx.x, gridDim.x);  // this CTA's rows: blockIdx.x + j*gridDim.x
  RingPos first;  // ring position of the current row's first tile
  // A flat row is inside the launch exactly when its matrix index is.
  for (int64_t j = 0; rows.inside(g); ++j, rows.next(g)) {
    const int64_t off = rows.offset(g);
    const int32_t valid = valid_cols(g, rows.i);
    const int32_t nvec = (valid + 7) >> 3;
    const int32_t nt = (nvec + tile_vec - 1) / tile_vec;
    const bool resident = nt <= S;
    // Vector v of the row, from lane slot lv of stage st; halves past the
    // causal boundary read as -inf (they lose the max and give exp 0).
    auto vec_at = [&](int st, int32_t v, int32_t lv) {
      uint4 r = *reinterpret_cast<const uint4*>(tiles + (size_t)st * tile_bytes + (size_t)lv * 16);
      const int32_t lim = valid - v * 8;
      if (lim < 8) r = mask_tail_neg_inf(r, lim);
      return r;
    };

    // Pass 1: this lane's online (max, sum); zero scale: its count of
    // elements that are not -inf.
    float m = -INFINITY;
    float2 acc = make_float2(0.f, 0.f);
    bool bad = false;  // a wait ran out: skip the rest of the row's waits
    RingPos pos = first;
    for (int32_t t = 0; t < nt; ++t, pos.next(S)) {
      const int st = pos.s;
      if (!bad && !mbar_wait_bounded(&full[st], pos.ph, g.timeout_ns)) {
        bad = true;
        *abort_flag = 1;
        if (g.status) atomicOr(g.status, kStatusTimeout);
      }
      if (!bad) {
#pragma unroll
        for (int q = 0; q < VPT; ++q) {
          const int32_t lv = q * 32 * W + lv0;
          const int32_t v = t * tile_vec + lv;
          if (v < nvec) {
            const uint4 r = vec_at(st, v, lv);
            const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
            if constexpr (kZeroScale) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                acc.x += (w4[e] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
                acc.y += (w4[e] >> 16) == kHalfNegInf ? 0.f : 1.f;
              }
            } else {
              const float vm = __half2float(max8_half(r));
              if (vm > m) {
                // (m - vm) * sl is -inf while m is -inf: the empty sum stays 0.
                const float c = ex2((m - vm) * sl);
                acc = __fmul2_rn(acc, make_float2(c, c));
                m = vm;
              }
              if (m > -INFINITY) {
                const float2 nm2 = make_float2(-m, -m);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w4[e])), nm2), sl2);
                  acc = __fadd2_rn(acc, make_float2(ex2(d.x), ex2(d.y)));
                }
              }
            }
          }
        }
      }
      if (!resident) {
        // Fetched again for pass 2: this warp is done with the stage.
        __syncwarp();
        if (lane == 0 && !bad) mbar_arrive(&empty[st]);
      }
    }

    // Row statistics: the warp's max (one redux instruction) and the sum of
    // its lanes' sums rescaled to it, then the same across the consumer warps.
    float s = acc.x + acc.y;
    if constexpr (!kZeroScale) {
      const float wm = redux_max(m);
      s = m > -INFINITY ? s * ex2((m - wm) * sl) : 0.f;
      m = wm;
    }
    s = warp_sum(s);
    float2* rk = red + (j & 1) * 32;  // two rows' slots: a warp runs at most one row ahead
    if (lane == 0) rk[warp] = make_float2(m, s);
    if (bar_red_or(1, W * 32, bad || *abort_flag != 0)) {
      *abort_flag = 1;
      break;
    }
    const float2 w = lane < W ? rk[lane] : make_float2(-INFINITY, 0.f);
    float rm = -INFINITY, rs;
    if constexpr (kZeroScale) {
      rs = warp_sum(w.y);
    } else {
      rm = redux_max(w.x);
      rs = warp_sum(w.x > -INFINITY ? w.y * ex2((w.x - rm) * sl) : 0.f);
    }
    const float inv = rcp_rn(rs);
    const float2 inv2 = make_float2(inv, inv);
    const float2 nM2 = make_float2(-rm, -rm);
    float lgs;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(lgs) : "f"(rs));
    const float2 nl2 = make_float2(-lgs, -lgs);

    // Pass 2: normalise and write; each tile's stage is handed back after it.
    uint16_t* out_row = g.out + off;
    if (resident) pos = first;  // the row's tiles again; else its second fetch follows
    for (int32_t t = 0; t < nt; ++t, pos.next(S)) {
      const int st = pos.s;
      if (!resident && !bad && !mbar_wait_bounded(&full[st], pos.ph, g.timeout_ns)) {
        bad = true;
        *abort_flag = 1;
        if (g.status) atomicOr(g.status, kStatusTimeout);
      }
      if (!bad) {
#pragma unroll
        for (int q = 0; q < VPT; ++q) {
          const int32_t lv = q * 32 * W + lv0;
          const int32_t v = t * tile_vec + lv;
          if (v < nvec) {
            const uint4 r = vec_at(st, v, lv);
            const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 x;
              if constexpr (kZeroScale) {
                x.x = (w4[e] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
                x.y = (w4[e] >> 16) == kHalfNegInf ? 0.f : 1.f;
              } else {
                const float2 d = __ffma2_rn(__fadd2_rn(__half22float2(bits_h2(w4[e])), nM2), sl2, nl2);
                x = make_float2(ex2(d.x), ex2(d.y));
              }
              const float2 pr = kZeroScale ? __fmul2_rn(x, inv2) : x;
              o[e] = float2_to_half2_bits(pr.x, pr.y);
            }
            *reinterpret_cast<uint4*>(out_row + (int64_t)v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0 && !bad) mbar_arrive(&empty[st]);
    }
    first = pos;
  }
}

template <int VPT>
__global__ void __launch_bounds__(1024, 1) online_kernel(const __grid_constant__ OnlineParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = (blockDim.x >> 5) - 1;  // consumer warps; warp W is the producer
  const int32_t tile_vec = 32 * W * VPT;
  const size_t tile_bytes = (size_t)tile_vec * 16;
  const int S = p.stages;
  uint8_t* tiles = smem;
  uint8_t* zero_buf = smem + (size_t)S * tile_bytes;
  float2* red = reinterpret_cast<float2*>(zero_buf + kOnlineZeroBytes);  // [2][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 64);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  const bool skip_loads = (g.flags & kFlagSkipLoads) != 0;
  const int32_t pv = g.pitch >> 3;

  for (int i = tid; i < kOnlineZeroBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(zero_buf)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();  // the zeros are visible to the bulk-store engine
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)W);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == W) {
    // ------------------------------------------------------------ producer
    if (lane != 0 || skip_loads) return;
    // The first S tiles' rows into L2 while the previous kernel in the stream
    // finishes (a prefetch consumes no data; L2 is where every write lands).
    {
      int32_t n = 0;
      RowCursor pre(g, blockIdx.x, gridDim.x);
      for (; pre.inside(g) && n < S; pre.next(g)) {
        const int64_t off = pre.offset(g);
        const int32_t nvec = (valid_cols(g, pre.i) + 7) >> 3;
        for (int32_t v0 = 0; v0 < nvec && n < S; v0 += tile_vec, ++n)
          bulk_prefetch_l2(g.in + off + (int64_t)v0 * 8, (uint32_t)min(tile_vec, nvec - v0) * 16u);
      }
    }
    pdl_wait();  // inputs written, outputs read by the previous kernel: done
    const uint64_t pol_first = policy_evict_first();
    bool aborted = false;
    int64_t li = 0;  // load index of the next copy
    RingPos pos;     // its ring position
    RowCursor rows(g, blockIdx.x, gridDim.x);  // this CTA's rows: blockIdx.x + j*gridDim.x
    for (; rows.inside(g) && !aborted; rows.next(g)) {
      const int64_t off = rows.offset(g);
      const int32_t nvec = (valid_cols(g, rows.i) + 7) >> 3;
      const int32_t nt = (nvec + tile_vec - 1) / tile_vec;
      const bool resident = nt <= S;
      // Masked columns and pitch padding: zeros, by bulk stores.
      for (int32_t z = nvec; z < pv; z += kOnlineZeroBytes / 16)
        bulk_s2g(g.out + off + (int64_t)z * 8, zero_buf, (uint32_t)min(kOnlineZeroBytes / 16, pv - z) * 16u);
      bulk_commit();
      bulk_wait_read_16();
      for (int pass = 0; pass < (resident ? 1 : 2) && !aborted; ++pass) {
        for (int32_t t = 0; t < nt; ++t, ++li, pos.next(S)) {
          const int s = pos.s;
          if (li >= S) {
            // The stage's previous use: the phase before the current one.
            if (!mbar_wait_bounded(&empty[s], pos.ph ^ 1u, g.timeout_ns)) {
              aborted = true;
              *abort_flag = 1;
              if (g.status) atomicOr(g.status, kStatusTimeout);
              break;
            }
            if (*abort_flag) {  // the consumers gave up
              aborted = true;
              break;
            }
          }
          const int32_t v0 = t * tile_vec;
          const uint32_t bytes = (uint32_t)min(tile_vec, nvec - v0) * 16u;
          mbar_arrive_expect_tx(&full[s], bytes);
          if (pass == 0)
            bulk_g2s(tiles + (size_t)s * tile_bytes, g.in + off + (int64_t)v0 * 8, bytes, &full[s]);
          else
            bulk_g2s_hint(tiles + (size_t)s * tile_bytes, g.in + off + (int64_t)v0 * 8, bytes, &full[s],
                          pol_first);
        }
      }
    }
    bulk_wait_all();
    // After an abort: let this CTA's copies in flight land (bounded).
    // Stage k's last use is d = (pos.s - 1 - k) mod S loads back, in the
    // current lap for k < pos.s and in the previous one otherwise.
    if (aborted)
      for (int k = 0; k < S; ++k) {
        const int d = (pos.s - 1 - k + S) % S;
        if (li - 1 - d < 0) continue;
        (void)mbar_wait_bounded(&full[k], k < pos.s ? pos.ph : pos.ph ^ 1u, g.timeout_ns);
      }
    return;
  }

  // ------------------------------------------------------------ consumers
  pdl_wait();  // their stores follow the previous kernel's reads
  if (g.scale * kLog2e == 0.f)
    online_consumers<VPT, true>(p, tiles, red, full, empty, abort_flag, warp, lane, W);
  else
    online_consumers<VPT, false>(p, tiles, red, full, empty, abort_flag, warp, lane, W);
}

}  // namespace cs
