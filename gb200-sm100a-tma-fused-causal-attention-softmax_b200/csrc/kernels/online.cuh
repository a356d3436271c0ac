// Pipelined online-softmax causal kernel for long rows (the `online` kernel
// choice, and the automatic choice once a row no longer fits the
// row-resident kernel's registers).
//
// Replaces gpu/src/main.rs:546-727 (two dense TMA passes, 2 KB tiles, one
// tile in flight per buffer, wait_group(0) after every store):
//
//  * each CTA owns whole rows (flat row index blockIdx.x + j*gridDim.x) and a
//    ring of S shared-memory tiles of VPT 16-byte vectors per thread (256
//    threads x 2 = 8 KB, or 1024 threads x 1 = 16 KB for long rows, so that a
//    row of up to ~114K columns stays resident and a whole SM works on it);
//    thread 0 keeps the ring full with 1-D TMA bulk copies of the causal
//    prefix only, running ahead across row boundaries;
//  * pass 1 keeps a per-thread online (max, sum) pair, merged at the end of
//    the row with warp-shuffle butterflies and one cross-warp exchange;
//  * pass 2 recomputes exp, scales by the reciprocal of the sum and writes
//    16-byte vectors straight from registers. When the row fits the ring it
//    stays resident in shared memory between the passes, so HBM sees a single
//    read, and pass 2 hands each tile back as soon as it is written out, so
//    the next row's tiles stream in while this row's go out; longer rows are
//    fetched again for pass 2 (the first fetch leaves them in L2 with a
//    normal priority, the second marks them evict-first);
//  * masked columns and padding are 16-byte zero stores.
//
// All mbarrier waits are bounded (Geometry::timeout_ns) and report
// kStatusTimeout through the status word.
#pragma once

#include "common.cuh"
#include "geometry.cuh"

namespace cs {

// Launch shapes: (threads, 16-byte vectors per thread and tile).
constexpr int kOnlineThreads = 256;  // the default shape: 8 KB tiles
constexpr int kOnlineVecPerThread = 2;
constexpr int kOnlineTileVec = kOnlineThreads * kOnlineVecPerThread;  // 512 vectors
constexpr int kOnlineTileBytes = kOnlineTileVec * 16;                 // 8 KB
constexpr int kOnlineWideThreads = 1024;  // long rows: 16 KB tiles, one vector per thread

struct OnlineParams {
  Geometry g;
  int64_t total_rows;  // batch * rows
  int32_t stages;      // ring depth (tiles of blockDim.x * VPT vectors)
};

__host__ __device__ constexpr int online_tail_bytes(int stages) { return 32 * 8 + stages * 8 + 16; }

// (m, s) merge of two online-softmax partial states.
// m are row maxima of the raw values; sl = scale*log2(e).
// An empty state has m == -inf; it is handled apart because (-inf - mn) * sl
// is NaN when the scale is 0.
__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2, float sl) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  const float mn = fmaxf(m, m2);
  s = s * ex2((m - mn) * sl) + s2 * ex2((m2 - mn) * sl);
  m = mn;
}

template <int VPT>
__global__ void __launch_bounds__(1024) online_kernel(const __grid_constant__ OnlineParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int n_warps = nthreads >> 5;
  const int32_t tile_vec = nthreads * VPT;             // vectors per tile
  const size_t tile_bytes = (size_t)tile_vec * 16;
  const int S = p.stages;
  uint8_t* tiles = smem;
  float2* red = reinterpret_cast<float2*>(smem + (size_t)S * tile_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 32);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + S);

  const int64_t G = gridDim.x;
  const int64_t n_rows = blockIdx.x < p.total_rows ? (p.total_rows - 1 - blockIdx.x) / G + 1 : 0;
  const bool skip_loads = (g.flags & kFlagSkipLoads) != 0;
  const int32_t pv = g.pitch >> 3;
  const float sl = g.scale * kLog2e;  // exponents (x - max) * scale*log2(e)

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // inputs written, outputs read by the previous kernel: done

  // Row j of this CTA -> element offset of its first column and valid count.
  auto row_of = [&](int64_t j, int64_t& off, int32_t& valid) {
    const int64_t flat = blockIdx.x + j * G;
    const int64_t b = flat / g.rows;
    const int32_t i = (int32_t)(flat - b * g.rows);
    off = b * g.batch_stride + (int64_t)i * g.pitch;
    valid = valid_cols(g, i);
  };

  // ---- producer state (meaningful in thread 0 only) ----
  int64_t loads = 0;     // copies issued so far (load index of the next copy)
  int64_t released = 0;  // copies whose stage has been handed back
  int64_t pj = 0;        // producer cursor: row, pass, tile
  int32_t ppass = 0, pt = 0;
  int64_t p_off = 0;
  int32_t p_nvec = 0, p_nt = 0;
  bool p_res = false;
  uint64_t pol_first = 0;
  if (tid == 0 && n_rows > 0) {
    int32_t valid;
    row_of(0, p_off, valid);
    p_nvec = (valid + 7) >> 3;
    p_nt = (p_nvec + tile_vec - 1) / tile_vec;
    p_res = p_nt <= S;
    pol_first = policy_evict_first();
  }
  auto produce = [&]() {
    if (skip_loads) return;
    while (loads - released < S && pj < n_rows) {
      const int s = (int)(loads % S);
      const int32_t v0 = pt * tile_vec;
      const int32_t nvt = min(tile_vec, p_nvec - v0);
      mbar_arrive_expect_tx(&full[s], (uint32_t)nvt * 16u);
      const uint16_t* src = g.in + p_off + (int64_t)v0 * 8;
      if (ppass == 0)
        bulk_g2s(tiles + (size_t)s * tile_bytes, src, (uint32_t)nvt * 16u, &full[s]);
      else
        bulk_g2s_hint(tiles + (size_t)s * tile_bytes, src, (uint32_t)nvt * 16u, &full[s], pol_first);
      ++loads;
      if (++pt == p_nt) {
        pt = 0;
        if (ppass == 0 && !p_res) {
          ppass = 1;
        } else {
          ppass = 0;
          if (++pj < n_rows) {
            int32_t valid;
            row_of(pj, p_off, valid);
            p_nvec = (valid + 7) >> 3;
            p_nt = (p_nvec + tile_vec - 1) / tile_vec;
            p_res = p_nt <= S;
          }
        }
      }
    }
  };
  if (tid == 0) produce();

  int64_t base = 0;  // load index of the current row's first tile (same in every thread)
  bool aborted = false;
  for (int64_t j = 0; j < n_rows && !aborted; ++j) {
    int64_t off;
    int32_t valid;
    row_of(j, off, valid);
    const int32_t nvec = (valid + 7) >> 3;
    const int32_t nt = (nvec + tile_vec - 1) / tile_vec;
    const bool resident = nt <= S;

    // Pass 1: online (max, sum) over this thread's vectors.
    float m = -INFINITY, s = 0.f;
    bool timed_out = false;  // after one expired wait, skip the rest of the row's waits
    for (int32_t t = 0; t < nt; ++t) {
      const int64_t idx = base + t;
      const int st = (int)(idx % S);
      if (timed_out || !mbar_wait_bounded(&full[st], (uint32_t)((idx / S) & 1), g.timeout_ns)) {
        if (!timed_out && g.status) atomicOr(g.status, kStatusTimeout);
        timed_out = true;
        *abort_flag = 1;
      } else {
#pragma unroll
        for (int q = 0; q < VPT; ++q) {
          const int32_t lv = tid + q * nthreads;  // vector within the tile
          const int32_t v = t * tile_vec + lv;    // vector within the row
          if (v < nvec) {
            const uint4 raw = *reinterpret_cast<const uint4*>(tiles + (size_t)st * tile_bytes + (size_t)lv * 16);
            const float2 f0 = half2_bits_to_float2(raw.x), f1 = half2_bits_to_float2(raw.y);
            const float2 f2 = half2_bits_to_float2(raw.z), f3 = half2_bits_to_float2(raw.w);
            const float z[8] = {f0.x, f0.y, f1.x, f1.y, f2.x, f2.y, f3.x, f3.y};
            const int32_t lim = valid - v * 8;
            float vm = -INFINITY;
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < lim) vm = fmaxf(vm, z[e]);
            const float mn = fmaxf(m, vm);
            float acc = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc += e < lim ? ex2((z[e] - mn) * sl) : 0.f;
            s = (m == -INFINITY ? 0.f : s * ex2((m - mn) * sl)) + acc;
            m = mn;
          }
        }
      }
      if (!resident) {
        __syncthreads();  // tile consumed by every thread
        if (*abort_flag) { aborted = true; break; }
        if (tid == 0) { released = idx + 1; produce(); }
      }
    }
    if (aborted) break;

    // Row statistics: warp butterflies of (m, s), then across warps.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2, sl);
    }
    if (lane == 0) red[warp] = make_float2(m, s);
    __syncthreads();
    if (*abort_flag) { aborted = true; break; }
    float2 w = lane < n_warps ? red[lane] : make_float2(-INFINITY, 0.f);
    float rm = w.x, rs = w.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, rm, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, rs, o);
      online_merge(rm, rs, m2, s2, sl);
    }
    const float inv = rcp_rn(rs);
    __syncthreads();  // red[] is rewritten by the next row

    // Pass 2: normalise and write.
    uint16_t* out_row = g.out + off;
    for (int32_t t = 0; t < nt; ++t) {
      const int64_t idx = resident ? base + t : base + nt + t;
      const int st = (int)(idx % S);
      bool ok = true;
      if (!resident) {
        ok = mbar_wait_bounded(&full[st], (uint32_t)((idx / S) & 1), g.timeout_ns);
        if (!ok) {
          *abort_flag = 1;
          if (g.status) atomicOr(g.status, kStatusTimeout);
        }
      }
      if (ok) {
#pragma unroll
        for (int q = 0; q < VPT; ++q) {
          const int32_t lv = tid + q * nthreads;
          const int32_t v = t * tile_vec + lv;
          if (v < nvec) {
            const uint4 raw = *reinterpret_cast<const uint4*>(tiles + (size_t)st * tile_bytes + (size_t)lv * 16);
            const float2 f0 = half2_bits_to_float2(raw.x), f1 = half2_bits_to_float2(raw.y);
            const float2 f2 = half2_bits_to_float2(raw.z), f3 = half2_bits_to_float2(raw.w);
            float z[8] = {f0.x, f0.y, f1.x, f1.y, f2.x, f2.y, f3.x, f3.y};
            const int32_t lim = valid - v * 8;
#pragma unroll
            for (int e = 0; e < 8; ++e) z[e] = e < lim ? ex2((z[e] - rm) * sl) * inv : 0.f;
            uint4 o;
            o.x = float2_to_half2_bits(z[0], z[1]);
            o.y = float2_to_half2_bits(z[2], z[3]);
            o.z = float2_to_half2_bits(z[4], z[5]);
            o.w = float2_to_half2_bits(z[6], z[7]);
            *reinterpret_cast<uint4*>(out_row + (int64_t)v * 8) = o;
          }
        }
      }
      // The tile is written out: hand its stage back (this row's next tiles
      // are already in their stages; the stage fills with a later tile).
      __syncthreads();
      if (*abort_flag) { aborted = true; break; }
      if (tid == 0) { released = idx + 1; produce(); }
    }
    if (aborted) break;
    base += resident ? nt : 2 * nt;

    for (int32_t v = nvec + tid; v < pv; v += nthreads)
      *reinterpret_cast<uint4*>(out_row + (int64_t)v * 8) = make_uint4(0u, 0u, 0u, 0u);
  }

  // After a timeout: let this CTA's copies in flight land (bounded).
  if (tid == 0 && aborted) {
    for (int64_t r = released; r < loads; ++r)
      (void)mbar_wait_bounded(&full[r % S], (uint32_t)((r / S) & 1), g.timeout_ns);
  }
}

}  // namespace cs
