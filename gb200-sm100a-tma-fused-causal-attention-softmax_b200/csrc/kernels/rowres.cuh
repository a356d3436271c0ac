// Row-resident single-pass causal softmax (the `tma` and `pipeline` kernel
// choices).
//
// Replaces the reference's three-pass TMA kernels (gpu/src/main.rs:202-541)
// with one read of the causal prefix and one write of the full row:
//
//  * persistent grid (SM count x resident CTAs) over the pair map in
//    geometry.cuh, so every unit carries the same number of causal elements;
//    CTA c starts with units c, c+G, ...; the register-resident variants keep
//    that static sequence, the shared-memory variant (V == 0) claims the
//    units after its first S from a per-plan counter (see the kernel);
//  * warp-specialised: one producer warp streams each unit's row prefixes
//    into a ring of shared-memory stages with 1-D TMA bulk copies
//    (cp.async.bulk, completing on a `full` mbarrier per stage) and writes the
//    masked columns and pitch padding with TMA bulk stores from a zeroed
//    shared buffer; only round_up(valid, 8) elements are ever read;
//  * register-resident consumers (V = 2, 4, 8) each own a contiguous segment
//    of ONE row (32*V 16-byte vectors, lane-interleaved so every load/store
//    instruction of a warp covers 512 contiguous bytes); a warp reduces its
//    own (max, sum) with redux.sync -- the max on packed halves (exact), the
//    exponents as (x - max) * scale*log2(e) with the Blackwell packed f32x2
//    add/mul, exp computed once per element with MUFU ex2 and kept in
//    registers -- and publishes it; after ONE named barrier per unit the
//    warps of a row merge the partials (online-softmax rescaling) and write
//    p = e * 2^((m_w - M)*scale*log2 e) / S; partials are double-buffered, so
//    one barrier suffices;
//  * shared-memory consumers (V = 0) leave the rows in the stage and make
//    three passes (max, sum, normalise) over their chunk, for rows too long
//    for registers (rowres_pass_consumers).
//
// With kTmaStore (`pipeline`) consumers write the normalised FP16 row back
// into the stage, and the producer warp sends it with TMA bulk stores
// (shared->global) before refilling the stage; without it (`tma`) consumers
// store from registers.
//
// Every mbarrier wait is bounded (Geometry::timeout_ns); on expiry the kernel
// sets kStatusTimeout in the status word, waits (bounded) for its own copies
// in flight and returns.
#pragma once

#include "common.cuh"
#include "geometry.cuh"

namespace cs {

constexpr int kZeroBytes = 4096;  // zero source of the bulk zero-fill stores

struct RowResParams {
  Geometry g;
  UnitMap m;
  int32_t stages;       // ring depth
  int32_t stage_bytes;  // bytes per stage (multiple of 128, >= 16 * max vectors per unit)
  int32_t l2_hint;      // 1: evict-first L2 hint on the input copies
  int32_t zero_tma;     // 1: masked columns by bulk stores, 0: by consumer stores
  int32_t prefetch;     // static units per CTA whose rows are pulled into L2 before the previous kernel ends
};

// Shared memory after the stages: zero buffer, 2 x 32 float2 (max, sum)
// partials, full and empty mbarriers per stage, abort flag, the unit each
// stage holds as its consumers see it (-1: no more units), and the
// producer's record of each stage's unit (matrix, in-matrix index) for its
// bulk stores -- in shared memory rather than a per-thread array, so that no
// kernel needs local memory.
__host__ __device__ constexpr int rowres_tail_bytes(int stages) {
  return kZeroBytes + 2 * 32 * 8 + 2 * stages * 8 + 16 + 3 * (((4 * stages + 15) / 16) * 16);
}

// Shared-memory-resident consumers (V == 0), for rows too long to hold in
// registers: each unit's rows stay in their ring stage and every consumer
// warp makes three passes over its contiguous chunk of one row -- the max,
// the sum of exp2((x - m_w) * scale*log2 e), and after the one barrier of the
// unit, p = exp2((x - M) * scale*log2 e) / S -- so a lane holds no row data
// between passes and 31 consumer warps fit one SM. Warps are given to the two
// rows of a pair in proportion to their lengths.
template <bool kTmaStore>
__device__ __forceinline__ void rowres_pass_consumers(const RowResParams& p, uint8_t* stage_base, float2* red,
                                                      uint64_t* full, uint64_t* empty,
                                                      volatile int* abort_flag, const volatile int32_t* unit_id,
                                                      int warp, int lane, int W) {
  const Geometry& g = p.g;
  const int S = p.stages;
  const int32_t upm = p.m.units_per_matrix;
  const int32_t pv = g.pitch >> 3;
  const float sl = g.scale * kLog2e;
  const float2 sl2 = make_float2(sl, sl);
  const bool zero_scale = sl == 0.f;
  int s = 0;
  uint32_t parity = 0;
  for (int32_t k = 0;; ++k) {
    // The producer names each stage's unit (possibly claimed at run time).
    const bool ok = mbar_wait_bounded(&full[s], parity, g.timeout_ns);
    if (!ok) {
      *abort_flag = 1;
      if (g.status) atomicOr(g.status, kStatusTimeout);
    }
    const int32_t u = ok ? unit_id[s] : 0;
    if (u < 0) break;
    const int32_t b = u / upm, kk = u - (u / upm) * upm;
    int32_t ra, rb;
    unit_rows(p.m, kk, ra, rb);
    const int32_t va = valid_cols(g, ra);
    const int32_t vb = rb >= 0 ? valid_cols(g, rb) : 0;
    const int32_t na = (va + 7) >> 3, nb = (vb + 7) >> 3;
    int32_t wa = W;
    if (nb > 0) {
      wa = (int32_t)(((int64_t)W * na + (na + nb) / 2) / (na + nb));
      wa = wa < 1 ? 1 : (wa > W - 1 ? W - 1 : wa);
    }
    const bool row_a = warp < wa;
    const int32_t w_first = row_a ? 0 : wa, w_count = row_a ? wa : W - wa;
    const int32_t n_row = row_a ? na : nb;
    const int32_t valid = row_a ? va : vb;
    // This warp's chunk: whole groups of 32 vectors, so lane j takes every
    // 32nd vector from c0 + j.
    const int32_t groups = (n_row + 31) >> 5;
    const int32_t per = (groups + w_count - 1) / w_count;
    const int32_t gs = (warp - w_first) * per;
    const int32_t c0 = (gs < groups ? gs : groups) * 32;
    const int32_t c1e = c0 + per * 32;
    const int32_t c1 = c1e < n_row ? c1e : n_row;
    uint8_t* st = stage_base + (size_t)s * p.stage_bytes + (size_t)(row_a ? 0 : na) * 16;
    constexpr uint32_t kNeg2 = kHalfNegInf | (kHalfNegInf << 16);
    auto load = [&](int32_t v) {
      uint4 r = *reinterpret_cast<const uint4*>(st + (size_t)v * 16);
      const int32_t lim = valid - v * 8;
      if (lim < 8) r = mask_tail_neg_inf(r, lim);
      return r;
    };
    // Pass 1: the warp's max (packed halves, exact).
    uint32_t hm = kNeg2;
    if (ok)
      for (int32_t v = c0 + lane; v < c1; v += 32) {
        const uint4 r = load(v);
        hm = h2_bits(__hmax2(bits_h2(hm), __hmax2(__hmax2(bits_h2(r.x), bits_h2(r.y)),
                                                   __hmax2(bits_h2(r.z), bits_h2(r.w)))));
      }
    const __half2 hm2 = bits_h2(hm);
    const float mw = redux_max(__half2float(__hmax(__low2half(hm2), __high2half(hm2))));
    // Pass 2: the warp's sum relative to its own max.
    float2 acc = make_float2(0.f, 0.f);
    if (ok && mw > -INFINITY) {
      const float2 nm2 = make_float2(-mw, -mw);
      for (int32_t v = c0 + lane; v < c1; v += 32) {
        const uint4 r = load(v);
        const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2 e;
          if (zero_scale) {
            e.x = (w4[q] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
            e.y = (w4[q] >> 16) == kHalfNegInf ? 0.f : 1.f;
          } else {
            const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w4[q])), nm2), sl2);
            e = make_float2(ex2(d.x), ex2(d.y));
          }
          acc = __fadd2_rn(acc, e);
        }
      }
    }
    const float sw = warp_sum(acc.x + acc.y);
    float2* rk = red + (k & 1) * 32;
    if (lane == 0) rk[warp] = make_float2(mw, sw);
    asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");  // consumer warps only
    if (*abort_flag) break;

    // Merge the row's warps: max M and sum S; then pass 3 writes exp2((x - M)*sl) / S.
    const float2 ps = lane < w_count ? rk[w_first + lane] : make_float2(-INFINITY, 0.f);
    const float M = redux_max(ps.x);
    const float Ssum = warp_sum(ps.x > -INFINITY ? ps.y * ex2((ps.x - M) * sl) : 0.f);
    const float rs = rcp_rn(Ssum);
    const float2 rs2 = make_float2(rs, rs);
    const float2 nM2 = make_float2(-M, -M);
    uint16_t* out_row = g.out + (int64_t)b * g.batch_stride + (int64_t)(row_a ? ra : rb) * g.pitch;
    for (int32_t v = c0 + lane; v < c1; v += 32) {
      const uint4 r = load(v);
      const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 e;
        if (zero_scale) {
          e.x = (w4[q] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
          e.y = (w4[q] >> 16) == kHalfNegInf ? 0.f : 1.f;
        } else {
          const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w4[q])), nM2), sl2);
          e = make_float2(ex2(d.x), ex2(d.y));
        }
        const float2 pr = __fmul2_rn(e, rs2);
        o[q] = float2_to_half2_bits(pr.x, pr.y);
      }
      const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
      if (kTmaStore)
        *reinterpret_cast<uint4*>(st + (size_t)v * 16) = ov;
      else
        *reinterpret_cast<uint4*>(out_row + (int64_t)v * 8) = ov;
    }
    if (kTmaStore) fence_proxy_async_smem();  // outputs visible to the bulk-store engine
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage
    if (!p.zero_tma && w_first == warp) {
      // Masked columns and pitch padding by the row's first warp (no loads).
      for (int32_t zi = n_row + lane; zi < pv; zi += 32)
        *reinterpret_cast<uint4*>(out_row + (int64_t)zi * 8) = make_uint4(0u, 0u, 0u, 0u);
    }
    if (++s == S) {
      s = 0;
      parity ^= 1u;
    }
  }
}

// V: 16-byte vectors per consumer lane (0: rows stay in shared memory, see
// rowres_pass_consumers); MAXT / MINB: launch bounds (CTA size and resident
// CTAs per SM), which set the register budget.
template <int V, int MAXT, int MINB, bool kTmaStore>
__global__ void __launch_bounds__(MAXT, MINB) rowres_kernel(const __grid_constant__ RowResParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = (blockDim.x >> 5) - 1;  // consumer warps; warp W is the producer
  const int S = p.stages;
  uint8_t* stage_base = smem;
  uint8_t* zero_buf = smem + (size_t)S * p.stage_bytes;
  float2* red = reinterpret_cast<float2*>(zero_buf + kZeroBytes);  // [2][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 64);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
  volatile int32_t* unit_id = reinterpret_cast<volatile int32_t*>(empty + S) + 4;

  // Schedule: CTA c takes units c, c + G, ..., c + (S-1) G; after those,
  // either the static sequence continues (c + S G, ...) or, with a schedule
  // counter (g.sched, set for the shared-memory consumers only), the producer
  // claims units from S G upwards one at a time, so CTAs that run ahead take
  // more. The producer names each stage's unit in unit_id and marks the end
  // with -1; the register-resident consumers follow the static sequence with
  // their own cursor, so a unit's geometry is ready before its data arrives.
  // The host splits launches so that total_units < 2^30.
  const int32_t G = gridDim.x;
  const int32_t first = blockIdx.x;
  const int32_t total = (int32_t)p.m.total_units;
  const int32_t upm = p.m.units_per_matrix;
  const int32_t gq = G / upm, gr = G - (G / upm) * upm;
  const bool skip_loads = (g.flags & kFlagSkipLoads) != 0;
  const int32_t pv = g.pitch >> 3;  // 16-byte vectors per output row
  const int32_t n_mine = first < total ? (total - 1 - first) / G + 1 : 0;
  // Only the shared-memory consumers read unit ids, so only they can follow claims.
  const bool claims = V == 0 && g.sched != nullptr;
  // Static units of this CTA (the rest, if any, are claimed).
  const int32_t n_static_mine = claims ? min(S, n_mine) : n_mine;
  const bool has_claims = claims && (int64_t)S * G < total;

  for (int i = tid; i < kZeroBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(zero_buf)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();  // zero buffer visible to the bulk-store engine
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
    const bool name_all = V == 0;  // consumers that read every stage's unit id
    // Unit held by each stage: matrix and in-matrix index (for its bulk stores).
    int32_t* sb = const_cast<int32_t*>(unit_id) + ((S + 3) & ~3);
    int32_t* sk = sb + ((S + 3) & ~3);
    // One unit's rows and 16-byte vector counts (computed once per unit).
    struct UnitGeo {
      int32_t b, kk, ra, rb;
      uint32_t na, nb;
    };
    auto geo = [&](int32_t b, int32_t kk) {
      UnitGeo u;
      u.b = b;
      u.kk = kk;
      unit_rows(p.m, kk, u.ra, u.rb);
      u.na = (uint32_t)(valid_cols(g, u.ra) + 7) >> 3;
      u.nb = u.rb >= 0 ? (uint32_t)(valid_cols(g, u.rb) + 7) >> 3 : 0u;
      return u;
    };
    // The static sequence first, first + G, ... as (matrix, in-matrix index)
    // cursors stepped without division.
    // kk and gr are below upm < 2^31, so their sum fits 32 unsigned bits.
    auto step = [&](int32_t& b, int32_t& kk) {
      uint32_t n = (uint32_t)kk + (uint32_t)gr;
      b += gq;
      if (n >= (uint32_t)upm) {
        n -= (uint32_t)upm;
        ++b;
      }
      kk = (int32_t)n;
    };
    // Masked columns and pitch padding of a unit: bulk stores from the zero buffer.
    auto zero_fill = [&](const UnitGeo& u) {
      uint16_t* out_m = g.out + (int64_t)u.b * g.batch_stride;
      for (int r = 0; r < 2; ++r) {
        const int32_t row = r == 0 ? u.ra : u.rb;
        if (row < 0) break;
        const uint32_t nv = r == 0 ? u.na : u.nb;
        uint8_t* z = reinterpret_cast<uint8_t*>(out_m + (int64_t)row * g.pitch + (int64_t)nv * 8);
        uint32_t left = (uint32_t)(pv - (int32_t)nv) * 16u;
        while (left) {
          const uint32_t n = left < (uint32_t)kZeroBytes ? left : (uint32_t)kZeroBytes;
          bulk_s2g(z, zero_buf, n);
          z += n;
          left -= n;
        }
      }
      bulk_commit();
      bulk_wait_read_16();
    };
    // kTmaStore: the output of the unit that last used a stage is stored
    // from it before the stage is refilled.
    auto store_unit = [&](int32_t ub, int32_t uk, int s) {
      const UnitGeo u = geo(ub, uk);
      uint16_t* out_m = g.out + (int64_t)ub * g.batch_stride;
      const uint8_t* st = stage_base + (size_t)s * p.stage_bytes;
      bulk_s2g(out_m + (int64_t)u.ra * g.pitch, st, u.na * 16u);
      if (u.nb) bulk_s2g(out_m + (int64_t)u.rb * g.pitch, st + (size_t)u.na * 16, u.nb * 16u);
      bulk_commit();
    };
    // Stage s receives unit u: its transaction bytes are announced first
    // (possibly before the previous kernel has finished), its copies are
    // issued only after that kernel has.
    auto announce = [&](const UnitGeo& u, int s) { mbar_arrive_expect_tx(&full[s], (u.na + u.nb) * 16u); };
    auto load = [&](const UnitGeo& u, int s) {
      uint8_t* dst = stage_base + (size_t)s * p.stage_bytes;
      const uint16_t* src = g.in + (int64_t)u.b * g.batch_stride;
      if (p.l2_hint) {
        const uint64_t policy = policy_evict_first();
        bulk_g2s_hint(dst, src + (int64_t)u.ra * g.pitch, u.na * 16u, &full[s], policy);
        if (u.nb) bulk_g2s_hint(dst + u.na * 16u, src + (int64_t)u.rb * g.pitch, u.nb * 16u, &full[s], policy);
      } else {
        bulk_g2s(dst, src + (int64_t)u.ra * g.pitch, u.na * 16u, &full[s]);
        if (u.nb) bulk_g2s(dst + u.na * 16u, src + (int64_t)u.rb * g.pitch, u.nb * 16u, &full[s]);
      }
    };

    int32_t lb = first / upm, lkk = first - (first / upm) * upm;  // next static unit to load
    // The first min(S, n_static_mine) units are static: announce them and
    // start pulling their rows into L2 before waiting for the previous kernel
    // (a prefetch consumes no data, and L2 is where every write lands, so
    // nothing stale can be read), then issue their copies at once.
    const int32_t n_pre = min(S, n_static_mine);
    for (int32_t k = 0; k < n_pre; ++k) {
      if (name_all) unit_id[k] = first + k * G;
      const UnitGeo u = geo(lb, lkk);
      announce(u, k);
      const uint16_t* src = g.in + (int64_t)u.b * g.batch_stride;
      bulk_prefetch_l2(src + (int64_t)u.ra * g.pitch, u.na * 16u);
      if (u.nb) bulk_prefetch_l2(src + (int64_t)u.rb * g.pitch, u.nb * 16u);
      sb[k] = lb;
      sk[k] = lkk;
      step(lb, lkk);
    }
    {
      // More of this CTA's static units, into L2 only.
      int32_t pb = lb, pk = lkk;
      for (int32_t k = n_pre; k < min(p.prefetch, n_static_mine); ++k) {
        const UnitGeo u = geo(pb, pk);
        const uint16_t* src = g.in + (int64_t)u.b * g.batch_stride;
        bulk_prefetch_l2(src + (int64_t)u.ra * g.pitch, u.na * 16u);
        if (u.nb) bulk_prefetch_l2(src + (int64_t)u.rb * g.pitch, u.nb * 16u);
        step(pb, pk);
      }
    }
    pdl_wait();  // inputs written, outputs read by the previous kernel: done
    for (int32_t k = 0; k < n_pre; ++k) {
      const UnitGeo u = geo(sb[k], sk[k]);
      load(u, k);
      if (p.zero_tma) zero_fill(u);
    }

    bool aborted = false;
    int32_t k = n_pre;  // also the number of units whose copies were issued, at every exit below
    // Units past the static part are claimed one iteration ahead, after that
    // iteration's copies, so the claim's L2 round trip overlaps them.
    auto claim = [&]() -> int32_t {
      const int64_t u = (int64_t)S * G + atomicAdd(&g.sched[0], 1u);
      return u < total ? (int32_t)u : -1;
    };
    int32_t next = k < n_static_mine ? 0 : (has_claims ? claim() : -1);  // the claimed unit, -1: none
    for (;; ++k) {
      const int s = k % S;
      if (k >= S) {
        if (!mbar_wait_bounded(&empty[s], (uint32_t)(((k / S) - 1) & 1), g.timeout_ns)) {
          aborted = true;
          *abort_flag = 1;
          if (g.status) atomicOr(g.status, kStatusTimeout);
          break;
        }
        if (kTmaStore) {
          store_unit(sb[s], sk[s], s);
          bulk_wait_read_all();  // the stage is read out before it is refilled
        }
      }
      const bool is_static = k < n_static_mine;
      if (!is_static && next < 0) {
        // End mark for the consumers that read unit ids.
        if (name_all) {
          unit_id[s] = -1;
          mbar_arrive(&full[s]);
        }
        break;
      }
      UnitGeo u;
      if (is_static) {
        u = geo(lb, lkk);
        step(lb, lkk);
        if (name_all) unit_id[s] = first + k * G;
      } else {
        u = geo(next / upm, next - (next / upm) * upm);
        unit_id[s] = next;
      }
      announce(u, s);
      load(u, s);
      if (p.zero_tma) zero_fill(u);
      sb[s] = u.b;
      sk[s] = u.kk;
      if (k + 1 >= n_static_mine) next = has_claims ? claim() : -1;
    }
    if (kTmaStore && !aborted) {
      // Outputs of the units still held by the other stages (iteration k
      // stored the one before it in its own stage).
      for (int32_t j = k + 1; j < k + S; ++j) {
        if (j - S < 0) continue;
        const int s = j % S;
        if (!mbar_wait_bounded(&empty[s], (uint32_t)(((j / S) - 1) & 1), g.timeout_ns)) {
          if (g.status) atomicOr(g.status, kStatusTimeout);
          break;
        }
        store_unit(sb[s], sk[s], s);
      }
    }
    if (claims) {
      // The last CTA to finish claiming resets the counters for the next launch.
      __threadfence();
      if (atomicAdd(&g.sched[1], 1u) == (uint32_t)G - 1) {
        atomicExch(&g.sched[0], 0u);
        atomicExch(&g.sched[1], 0u);
      }
    }
    bulk_wait_all();
    // After an abort: copies this warp issued that no consumer waited for.
    // (Without one, every copy was consumed, and a stage that received the
    // end mark has completed one more phase, so its parity no longer tells.)
    if (aborted)
      for (int32_t r = (k > S ? k - S : 0); r < k; ++r)
        (void)mbar_wait_bounded(&full[r % S], (uint32_t)((r / S) & 1), g.timeout_ns);
    return;
  }

  pdl_wait();  // consumers store to global memory (outputs, thread zero-fill)
  // -------------------------------------------------------------- consumers
  if constexpr (V == 0) {
    rowres_pass_consumers<kTmaStore>(p, stage_base, red, full, empty, abort_flag, unit_id, warp, lane, W);
  } else {
  const float sl = g.scale * kLog2e;  // exponents (x - max) * scale*log2(e)
  const float2 sl2 = make_float2(sl, sl);
  constexpr int kSeg = 32 * V;  // vectors per warp segment
  int32_t b = first / upm, kk = first - (first / upm) * upm;
  int s = 0;
  uint32_t parity = 0;
  for (int32_t k = 0; k < n_mine; ++k) {
    int32_t ra, rb;
    unit_rows(p.m, kk, ra, rb);
    const int32_t va = valid_cols(g, ra);
    const int32_t vb = rb >= 0 ? valid_cols(g, rb) : 0;
    const int32_t na = (va + 7) >> 3, nb = (vb + 7) >> 3;
    const int32_t wa = (na + kSeg - 1) / kSeg, wb = (nb + kSeg - 1) / kSeg;
    // This warp's row and segment (warps past wa + wb sit this unit out).
    const bool row_a = warp < wa;
    const bool active = warp < wa + wb;
    const int32_t seg = row_a ? warp : warp - wa;
    const int32_t n_row = row_a ? na : nb;
    const int32_t valid = row_a ? va : vb;
    const int32_t v0 = seg * kSeg + lane;  // this lane's first vector within the row

    const bool ok = mbar_wait_bounded(&full[s], parity, g.timeout_ns);
    if (!ok) {
      *abort_flag = 1;
      if (g.status) atomicOr(g.status, kStatusTimeout);
    }
    const uint8_t* st = stage_base + (size_t)s * p.stage_bytes + (size_t)(row_a ? 0 : na) * 16;

    // Vector slot j is skipped by the whole warp when its first lane is past
    // the row (a warp-uniform test). Lanes past the row's end in the last
    // slot, and the masked elements of the row's last vector, hold -inf
    // halves: they lose the max and give exp 0 with no further masking.
    const int32_t seg_first = seg * kSeg;  // warp-uniform
    constexpr uint32_t kNeg2 = kHalfNegInf | (kHalfNegInf << 16);
    uint4 raw[V];
    __half hm = __ushort_as_half((unsigned short)kHalfNegInf);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      raw[j] = make_uint4(kNeg2, kNeg2, kNeg2, kNeg2);
      if (ok && active && seg_first + 32 * j < n_row) {
        const int32_t v = v0 + 32 * j;
        const int32_t lim = valid - v * 8;  // <= 0 past the row's end
        if (lim > 0) raw[j] = *reinterpret_cast<const uint4*>(st + (size_t)v * 16);
        if (lim < 8) raw[j] = mask_tail_neg_inf(raw[j], lim);
        hm = __hmax(hm, max8_half(raw[j]));
      }
    }
    if (!kTmaStore) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // this warp's vectors are in registers
    }
    // Warp max (one redux instruction), then exp2 relative to it and the warp sum.
    const float mw = redux_max(__half2float(hm));
    const float2 nm2 = make_float2(-mw, -mw);
    float e[V][8];
    float2 acc = make_float2(0.f, 0.f);
    if (sl != 0.f) {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        if (active && seg_first + 32 * j < n_row) {
          const uint32_t w4[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // -inf halves: (-inf - mw) * sl = -inf for sl > 0, so exp is 0.
            const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w4[q])), nm2), sl2);
            e[j][2 * q] = ex2(d.x);
            e[j][2 * q + 1] = ex2(d.y);
          }
          acc = __fadd2_rn(acc, __fadd2_rn(__fadd2_rn(make_float2(e[j][0], e[j][1]), make_float2(e[j][2], e[j][3])),
                                           __fadd2_rn(make_float2(e[j][4], e[j][5]), make_float2(e[j][6], e[j][7]))));
        }
      }
    } else {
      // Zero scale: every causal element is exp(0) = 1 (uniform distribution).
#pragma unroll
      for (int j = 0; j < V; ++j) {
        if (active && seg_first + 32 * j < n_row) {
          const uint32_t w4[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            e[j][2 * q] = (w4[q] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
            e[j][2 * q + 1] = (w4[q] >> 16) == kHalfNegInf ? 0.f : 1.f;
          }
          acc = __fadd2_rn(acc, __fadd2_rn(__fadd2_rn(make_float2(e[j][0], e[j][1]), make_float2(e[j][2], e[j][3])),
                                           __fadd2_rn(make_float2(e[j][4], e[j][5]), make_float2(e[j][6], e[j][7]))));
        }
      }
    }
    // A lane's partial sum is at most 8V <= 64: 25 fractional bits fit.
    const float sw = warp_sum_fixed<25>(acc.x + acc.y);
    float2* rk = red + (k & 1) * 32;
    if (lane == 0) rk[warp] = active ? make_float2(mw, sw) : make_float2(-INFINITY, 0.f);
    asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");  // consumer warps only
    if (*abort_flag) break;

    // Merge the partials of this row's warps (lane i holds warp i's): the
    // row max M, the rescaled sum S, and this warp's factor 2^((mw-M)sl)/S.
    const int32_t w_first = row_a ? 0 : wa, w_count = row_a ? wa : wb;
    const float2 ps = lane < w_count ? rk[w_first + lane] : make_float2(-INFINITY, 0.f);
    const float M = redux_max(ps.x);
    // A warp's sum is at most 32 * 64 = 2^11: 20 fractional bits fit.
    const float Ssum = warp_sum_fixed<20>(lane < w_count ? ps.y * ex2((ps.x - M) * sl) : 0.f);
    const float c = ex2((mw - M) * sl) * rcp_rn(Ssum);
    const float2 c2 = make_float2(c, c);

    uint16_t* out_row = g.out + (int64_t)b * g.batch_stride + (int64_t)(row_a ? ra : rb) * g.pitch;
    uint8_t* st_out = stage_base + (size_t)s * p.stage_bytes + (size_t)(row_a ? 0 : na) * 16;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (active && seg_first + 32 * j < n_row) {
        const int32_t v = v0 + 32 * j;
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 pr = __fmul2_rn(make_float2(e[j][2 * q], e[j][2 * q + 1]), c2);
          o[q] = float2_to_half2_bits(pr.x, pr.y);
        }
        const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
        if (v < n_row) {
          if (kTmaStore)
            *reinterpret_cast<uint4*>(st_out + (size_t)v * 16) = ov;
          else
            *reinterpret_cast<uint4*>(out_row + (int64_t)v * 8) = ov;
        }
      }
    }
    if (kTmaStore) {
      fence_proxy_async_smem();  // outputs visible to the bulk-store engine
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!p.zero_tma) {
      // Masked columns and pitch padding by this warp's lanes (no loads).
      if (active && seg == 0) {
        for (int32_t zi = n_row + lane; zi < pv; zi += 32)
          *reinterpret_cast<uint4*>(out_row + (int64_t)zi * 8) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    {  // next static unit; kk + gr < 2 * upm < 2^32 in unsigned arithmetic
      uint32_t n = (uint32_t)kk + (uint32_t)gr;
      b += gq;
      if (n >= (uint32_t)upm) {
        n -= (uint32_t)upm;
        ++b;
      }
      kk = (int32_t)n;
    }
    if (++s == S) {
      s = 0;
      parity ^= 1u;
    }
  }
  }  // V > 0
}

}  // namespace cs
