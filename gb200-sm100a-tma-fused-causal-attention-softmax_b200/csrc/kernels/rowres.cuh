// Row-resident single-pass causal softmax (the `tma` kernel choice).
//
// Replaces the reference's three-pass TMA kernels (gpu/src/main.rs:202-541)
// with one read of the causal prefix and one write of the full row:
//
//  * persistent grid (SM count x resident CTAs); CTA c takes work units
//    c, c+G, c+2G, ... of the pair map in geometry.cuh, so every unit carries
//    the same number of causal elements and the schedule is balanced statically;
//  * one elected thread streams each unit's row prefixes into a ring of
//    shared-memory stages with 1-D TMA bulk copies (cp.async.bulk) completing
//    on one mbarrier per stage; only round_up(valid, 8) elements are fetched,
//    so the masked upper triangle is never read;
//  * every thread moves its V 16-byte vectors from the stage into registers;
//    the stage goes back to the producer at the first CTA barrier, so the
//    next copies overlap this unit's arithmetic;
//  * the row maximum is taken on packed halves (exact); each exponent is
//    (x - max) * scale*log2(e) -- exactly 0 for the maximum and its ties --
//    and exp is computed once per element (MUFU ex2) and kept in registers;
//    the Blackwell packed-f32 instructions (add/mul .f32x2) halve the
//    subtraction, scaling, summation and normalisation work; only a row's
//    last vector needs masking;
//  * max and sum are warp butterflies plus one cross-warp exchange each,
//    for both rows of a pair at once;
//  * the masked columns and pitch padding are written by TMA bulk stores
//    from a zeroed shared-memory buffer (no loads, no per-thread stores).
//
// The `pipeline` kernel choice is the same kernel with kTmaStore: the
// normalised FP16 row is written back into its stage and leaves through 1-D
// TMA bulk stores (cp.async.bulk shared->global), and a stage is refilled
// one unit later, once its bulk store has finished reading it.
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
  int32_t zero_tma;     // 1: masked columns by bulk stores, 0: by thread stores
};

// Shared memory after the stages: the zero buffer, 32 packed-half maxima,
// 32 float2 sums, one mbarrier per stage and an abort flag.
__host__ __device__ constexpr int rowres_tail_bytes(int stages) {
  return kZeroBytes + 32 * 4 + 32 * 8 + stages * 8 + 16;
}

template <int V, int MAXT, bool kTmaStore>
__global__ void __launch_bounds__(MAXT) rowres_kernel(const __grid_constant__ RowResParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int T = blockDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = T >> 5;
  const int S = p.stages;
  uint8_t* stage_base = smem;
  uint8_t* zero_buf = smem + (size_t)S * p.stage_bytes;
  uint32_t* red_max = reinterpret_cast<uint32_t*>(zero_buf + kZeroBytes);
  float2* red_sum = reinterpret_cast<float2*>(red_max + 32);
  uint64_t* full = reinterpret_cast<uint64_t*>(red_sum + 32);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + S);

  // Unit indices fit in 32 bits: the host splits launches so that
  // total_units < 2^30. Units advance by G per step; (matrix, unit) cursors
  // are stepped incrementally instead of divided.
  const int32_t G = gridDim.x;
  const int32_t first = blockIdx.x;
  const int32_t total = (int32_t)p.m.total_units;
  const int32_t n_mine = first < total ? (total - 1 - first) / G + 1 : 0;
  const int32_t upm = p.m.units_per_matrix;
  const int32_t gq = G / upm, gr = G - (G / upm) * upm;
  auto advance = [&](int32_t& b, int32_t& k) {
    k += gr;
    b += gq;
    if (k >= upm) {
      k -= upm;
      ++b;
    }
  };
  int32_t cb = first / upm, ck = first - (first / upm) * upm;  // consumer cursor
  int32_t pb = cb, pk = ck;                                    // producer cursor (thread 0)
  const bool skip_loads = (g.flags & kFlagSkipLoads) != 0;

  for (int i = tid; i < kZeroBytes / 16; i += T)
    reinterpret_cast<uint4*>(zero_buf)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();  // zero buffer visible to the bulk-store engine
  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // Producer (thread 0): fetch the causal prefixes of the next unit into stage s.
  uint64_t policy = 0;
  int32_t n_issued = 0;
  auto issue_next = [&](int s) {
    int32_t ra, rb;
    unit_rows(p.m, pk, ra, rb);
    const uint32_t va_vec = (uint32_t)(valid_cols(g, ra) + 7) >> 3;
    const uint32_t vb_vec = rb >= 0 ? (uint32_t)(valid_cols(g, rb) + 7) >> 3 : 0u;
    uint8_t* dst = stage_base + (size_t)s * p.stage_bytes;
    const uint16_t* src = g.in + (int64_t)pb * g.batch_stride;
    mbar_arrive_expect_tx(&full[s], (va_vec + vb_vec) * 16u);
    if (p.l2_hint) {
      bulk_g2s_hint(dst, src + (int64_t)ra * g.pitch, va_vec * 16u, &full[s], policy);
      if (vb_vec) bulk_g2s_hint(dst + va_vec * 16u, src + (int64_t)rb * g.pitch, vb_vec * 16u, &full[s], policy);
    } else {
      bulk_g2s(dst, src + (int64_t)ra * g.pitch, va_vec * 16u, &full[s]);
      if (vb_vec) bulk_g2s(dst + va_vec * 16u, src + (int64_t)rb * g.pitch, vb_vec * 16u, &full[s]);
    }
    advance(pb, pk);
    ++n_issued;
  };
  // Zero columns [from_vec, pitch) of a row with bulk stores of the zero buffer.
  const int32_t pv = g.pitch >> 3;  // 16-byte vectors per output row
  auto zero_fill = [&](uint16_t* row, int32_t from_vec) {
    uint8_t* dst = reinterpret_cast<uint8_t*>(row + (int64_t)from_vec * 8);
    uint32_t left = (uint32_t)(pv - from_vec) * 16u;
    while (left) {
      const uint32_t n = left < (uint32_t)kZeroBytes ? left : (uint32_t)kZeroBytes;
      bulk_s2g(dst, zero_buf, n);
      dst += n;
      left -= n;
    }
  };

  if (tid == 0 && !skip_loads) {
    if (p.l2_hint) policy = policy_evict_first();
    const int32_t pro = n_mine < S ? n_mine : S;
    for (int32_t k = 0; k < pro; ++k) issue_next(k);
  }

  const float sl = g.scale * kLog2e;  // logits in base 2
  const float2 sl2 = make_float2(sl, sl);
  int32_t k = 0;
  int s = 0;            // k % S
  uint32_t parity = 0;  // (k / S) & 1
  for (; k < n_mine; ++k, s = (s + 1 == S) ? 0 : s + 1, parity ^= (s == 0)) {
    int32_t ra, rb;
    unit_rows(p.m, ck, ra, rb);
    const int32_t va = valid_cols(g, ra);
    const int32_t vb = rb >= 0 ? valid_cols(g, rb) : 0;
    const int32_t na = (va + 7) >> 3;
    const int32_t nb = (vb + 7) >> 3;
    const int32_t nv = na + nb;

    const bool ok = mbar_wait_bounded(&full[s], parity, g.timeout_ns);
    if (!ok) {
      *abort_flag = 1;
      if (g.status) atomicOr(g.status, kStatusTimeout);
    }
    const uint8_t* st = stage_base + (size_t)s * p.stage_bytes;

    // Stage -> registers; row maxima on packed halves (masked tail = -inf).
    uint4 raw[V];
    __half ma = __ushort_as_half((unsigned short)kHalfNegInf);
    __half mb = ma;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int v = tid + j * T;
      raw[j] = make_uint4(0u, 0u, 0u, 0u);
      if (ok && v < nv) {
        raw[j] = *reinterpret_cast<const uint4*>(st + (size_t)v * 16);
        const bool in_a = v < na;
        const int32_t lim = in_a ? va - v * 8 : vb - (v - na) * 8;
        const __half mm = max8_half(lim < 8 ? mask_tail_neg_inf(raw[j], lim) : raw[j]);
        if (in_a) ma = __hmax(ma, mm); else mb = __hmax(mb, mm);
      }
    }
    uint32_t mab = warp_max_h2(h2_bits(__halves2half2(ma, mb)));
    if (lane == 0) red_max[warp] = mab;
    __syncthreads();  // stage s fully consumed; partial maxima published
    if (*abort_flag) break;

    uint16_t* out_m = g.out + (int64_t)cb * g.batch_stride;
    uint16_t* row_a = out_m + (int64_t)ra * g.pitch;
    uint16_t* row_b = rb >= 0 ? out_m + (int64_t)rb * g.pitch : row_a;
    if (tid == 0) {
      if (!skip_loads) {
        if (!kTmaStore) {
          if (n_issued < n_mine) issue_next(s);
        } else if (k >= 1 && n_issued < n_mine) {
          bulk_wait_read_all();  // unit k-1's bulk store has left its stage
          issue_next(s == 0 ? S - 1 : s - 1);
        }
      }
      if (p.zero_tma) {
        zero_fill(row_a, na);
        if (rb >= 0) zero_fill(row_b, nb);
        bulk_commit();
        bulk_wait_read_16();
      }
    }

    mab = lane < nwarps ? red_max[lane] : (kHalfNegInf | (kHalfNegInf << 16));
    mab = warp_max_h2(mab);
    const float2 mf = __half22float2(bits_h2(mab));  // row maxima of the halves

    // exp2((x - max) * scale*log2(e)) once per element, kept in registers.
    // The difference comes first: it is 0 for the maximum (and for its ties)
    // whatever the scale, and a product-then-subtract form would let the
    // compiler fuse it into one FMA that keeps the product's rounding residual.
    float e[V][8];
    float2 sa = make_float2(0.f, 0.f), sb = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int v = tid + j * T;
      if (v < nv) {
        const bool in_a = v < na;
        const int32_t lim = in_a ? va - v * 8 : vb - (v - na) * 8;
        const float nm = in_a ? -mf.x : -mf.y;
        const float2 nm2 = make_float2(nm, nm);
        const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w[q])), nm2), sl2);
          e[j][2 * q] = ex2(d.x);
          e[j][2 * q + 1] = ex2(d.y);
        }
        if (lim < 8) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (q >= lim) e[j][q] = 0.f;
        }
        const float2 acc = __fadd2_rn(__fadd2_rn(make_float2(e[j][0], e[j][1]), make_float2(e[j][2], e[j][3])),
                                      __fadd2_rn(make_float2(e[j][4], e[j][5]), make_float2(e[j][6], e[j][7])));
        if (in_a) sa = __fadd2_rn(sa, acc); else sb = __fadd2_rn(sb, acc);
      }
    }
    float2 sm = warp_sum2(make_float2(sa.x + sa.y, sb.x + sb.y));
    if (lane == 0) red_sum[warp] = sm;
    __syncthreads();  // partial sums published
    float2 q = lane < nwarps ? red_sum[lane] : make_float2(0.f, 0.f);
    q = warp_sum2(q);
    const float inv_a = rcp_rn(q.x);
    const float inv_b = rcp_rn(q.y);

#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int v = tid + j * T;
      if (v < nv) {
        const bool in_a = v < na;
        const float inv = in_a ? inv_a : inv_b;
        const float2 inv2 = make_float2(inv, inv);
        uint32_t o[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 pr = __fmul2_rn(make_float2(e[j][2 * c], e[j][2 * c + 1]), inv2);
          o[c] = float2_to_half2_bits(pr.x, pr.y);
        }
        const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
        if (kTmaStore) {
          *reinterpret_cast<uint4*>(stage_base + (size_t)s * p.stage_bytes + (size_t)v * 16) = ov;
        } else {
          uint16_t* dst = in_a ? row_a + (int64_t)v * 8 : row_b + (int64_t)(v - na) * 8;
          *reinterpret_cast<uint4*>(dst) = ov;
        }
      }
    }
    if (kTmaStore) {
      fence_proxy_async_smem();  // make this thread's stage writes visible to the bulk copy
      __syncthreads();
      if (tid == 0) {
        uint8_t* st_out = stage_base + (size_t)s * p.stage_bytes;
        bulk_s2g(row_a, st_out, (uint32_t)na * 16u);
        if (rb >= 0) bulk_s2g(row_b, st_out + (size_t)na * 16, (uint32_t)nb * 16u);
        bulk_commit();
      }
    }
    if (!p.zero_tma) {
      // Masked columns and pitch padding: 16-byte zero stores, no loads.
      const int32_t za = pv - na;
      const int32_t zb = rb >= 0 ? pv - nb : 0;
      for (int32_t zi = tid; zi < za + zb; zi += T) {
        uint16_t* dst = zi < za ? row_a + (int64_t)(na + zi) * 8 : row_b + (int64_t)(nb + zi - za) * 8;
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    advance(cb, ck);
  }

  // Bulk stores must finish reading shared memory before the CTA exits.
  if ((kTmaStore || p.zero_tma) && tid == 0) bulk_wait_all();

  // After a timeout: let this CTA's own copies in flight land (bounded)
  // before the shared memory they target is released.
  if (tid == 0 && k < n_mine) {
    for (int32_t r = k; r < n_issued; ++r)
      (void)mbar_wait_bounded(&full[r % S], (uint32_t)((r / S) & 1), g.timeout_ns);
  }
}

}  // namespace cs
