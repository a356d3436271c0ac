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
//  * every thread moves its 16-byte vectors from the stage into registers
//    (V vectors = 8V values per thread), and the stage is handed back to the
//    producer after the first CTA barrier, so the next loads overlap compute;
//  * max and sum are warp butterflies plus one cross-warp exchange each,
//    for both rows of a pair at once (float2); exp is computed once per
//    element (MUFU ex2) and kept in registers until the normalised FP16
//    values are written with 16-byte stores;
//  * the masked columns (and pitch padding) are written as 16-byte zero stores.
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

struct RowResParams {
  Geometry g;
  UnitMap m;
  int32_t stages;       // ring depth
  int32_t stage_bytes;  // bytes per stage (multiple of 128, >= 16 * max vectors per unit)
  int32_t l2_hint;      // 1: evict-first L2 hint on the input copies
};

// Shared memory after the stages: 64 float2 reduction slots, one mbarrier per
// stage and an abort flag.
__host__ __device__ constexpr int rowres_tail_bytes(int stages) { return 64 * 8 + stages * 8 + 16; }

template <int V, int MAXT, bool kTmaStore>
__global__ void __launch_bounds__(MAXT) rowres_kernel(const __grid_constant__ RowResParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int T = blockDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = T >> 5;
  const int S = p.stages;
  uint8_t* stage_base = smem;
  float2* red = reinterpret_cast<float2*>(smem + (size_t)S * p.stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 64);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + S);

  // Unit indices fit in 32 bits: the host splits launches so that
  // total_units < 2^31.
  const int32_t G = gridDim.x;
  const int32_t first = blockIdx.x;
  const int32_t total = (int32_t)p.m.total_units;
  const int32_t n_mine = first < total ? (total - 1 - first) / G + 1 : 0;
  const int32_t upm = p.m.units_per_matrix;
  const bool skip_loads = (g.flags & kFlagSkipLoads) != 0;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // Producer (thread 0): fetch the causal prefixes of local unit k into stage s.
  uint64_t policy = 0;
  int32_t n_issued = 0;
  auto issue = [&](int32_t k, int s) {
    const int32_t u = first + k * G;
    const int32_t b = u / upm;
    int32_t ra, rb;
    unit_rows(p.m, u - b * upm, ra, rb);
    const uint32_t va_vec = (uint32_t)(valid_cols(g, ra) + 7) >> 3;
    const uint32_t vb_vec = rb >= 0 ? (uint32_t)(valid_cols(g, rb) + 7) >> 3 : 0u;
    uint8_t* dst = stage_base + (size_t)s * p.stage_bytes;
    const uint16_t* src = g.in + (int64_t)b * g.batch_stride;
    mbar_arrive_expect_tx(&full[s], (va_vec + vb_vec) * 16u);
    if (p.l2_hint) {
      bulk_g2s_hint(dst, src + (int64_t)ra * g.pitch, va_vec * 16u, &full[s], policy);
      if (vb_vec) bulk_g2s_hint(dst + va_vec * 16u, src + (int64_t)rb * g.pitch, vb_vec * 16u, &full[s], policy);
    } else {
      bulk_g2s(dst, src + (int64_t)ra * g.pitch, va_vec * 16u, &full[s]);
      if (vb_vec) bulk_g2s(dst + va_vec * 16u, src + (int64_t)rb * g.pitch, vb_vec * 16u, &full[s]);
    }
    n_issued = k + 1;
  };

  if (tid == 0 && !skip_loads) {
    if (p.l2_hint) policy = policy_evict_first();
    const int32_t pro = n_mine < S ? n_mine : S;
    for (int32_t k = 0; k < pro; ++k) issue(k, k);
  }

  const float scale = g.scale;
  const int32_t pv = g.pitch >> 3;  // 16-byte vectors per output row
  int32_t k = 0;
  int s = 0;             // k % S
  uint32_t parity = 0;   // (k / S) & 1
  for (; k < n_mine; ++k, s = (s + 1 == S) ? 0 : s + 1, parity ^= (s == 0)) {
    const int32_t u = first + k * G;
    const int32_t b = u / upm;
    int32_t ra, rb;
    unit_rows(p.m, u - b * upm, ra, rb);
    const int32_t va = valid_cols(g, ra);
    const int32_t vb = rb >= 0 ? valid_cols(g, rb) : 0;
    const int32_t na = (va + 7) >> 3;
    const int32_t nv = na + ((vb + 7) >> 3);

    const bool ok = mbar_wait_bounded(&full[s], parity, g.timeout_ns);
    if (!ok) {
      *abort_flag = 1;
      if (g.status) atomicOr(g.status, kStatusTimeout);
    }
    const uint8_t* st = stage_base + (size_t)s * p.stage_bytes;

    // Stage -> registers; scaled logits with masked slots at -inf.
    float z[V][8];
    float2 mx = make_float2(-INFINITY, -INFINITY);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int v = tid + j * T;
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (ok && v < nv) raw = *reinterpret_cast<const uint4*>(st + (size_t)v * 16);
      const bool in_a = v < na;
      const int32_t lim = v < nv ? (in_a ? va - v * 8 : vb - (v - na) * 8) : 0;
      const float2 f0 = half2_bits_to_float2(raw.x), f1 = half2_bits_to_float2(raw.y);
      const float2 f2 = half2_bits_to_float2(raw.z), f3 = half2_bits_to_float2(raw.w);
      z[j][0] = f0.x * scale; z[j][1] = f0.y * scale;
      z[j][2] = f1.x * scale; z[j][3] = f1.y * scale;
      z[j][4] = f2.x * scale; z[j][5] = f2.y * scale;
      z[j][6] = f3.x * scale; z[j][7] = f3.y * scale;
      float vm = -INFINITY;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (e >= lim) z[j][e] = -INFINITY;
        vm = fmaxf(vm, z[j][e]);
      }
      if (in_a) mx.x = fmaxf(mx.x, vm); else mx.y = fmaxf(mx.y, vm);
    }
    mx = warp_max2(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();  // stage s fully consumed; partial maxima published
    if (*abort_flag) break;
    if (tid == 0 && !skip_loads) {
      if (!kTmaStore) {
        if (k + S < n_mine) issue(k + S, s);
      } else if (k >= 1 && k - 1 + S < n_mine) {
        bulk_wait_read_all();  // unit k-1's bulk store has left its stage
        issue(k - 1 + S, s == 0 ? S - 1 : s - 1);
      }
    }

    float2 t = lane < nwarps ? red[lane] : make_float2(-INFINITY, -INFINITY);
    t = warp_max2(t);

    float2 sm = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int v = tid + j * T;
      if (v < nv) {
        const bool in_a = v < na;
        const float m = in_a ? t.x : t.y;
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          z[j][e] = ex2((z[j][e] - m) * kLog2e);  // masked: ex2(-inf) = +0
          acc += z[j][e];
        }
        if (in_a) sm.x += acc; else sm.y += acc;
      }
    }
    sm = warp_sum2(sm);
    if (lane == 0) red[32 + warp] = sm;
    __syncthreads();  // partial sums published
    float2 q = lane < nwarps ? red[32 + lane] : make_float2(0.f, 0.f);
    q = warp_sum2(q);
    const float inv_a = rcp_rn(q.x);
    const float inv_b = rcp_rn(q.y);

    uint16_t* out_m = g.out + (int64_t)b * g.batch_stride;
    uint16_t* row_a = out_m + (int64_t)ra * g.pitch;
    uint16_t* row_b = rb >= 0 ? out_m + (int64_t)rb * g.pitch : row_a;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int v = tid + j * T;
      if (v < nv) {
        const bool in_a = v < na;
        const float inv = in_a ? inv_a : inv_b;
        uint4 o;
        o.x = float2_to_half2_bits(z[j][0] * inv, z[j][1] * inv);
        o.y = float2_to_half2_bits(z[j][2] * inv, z[j][3] * inv);
        o.z = float2_to_half2_bits(z[j][4] * inv, z[j][5] * inv);
        o.w = float2_to_half2_bits(z[j][6] * inv, z[j][7] * inv);
        if (kTmaStore) {
          *reinterpret_cast<uint4*>(stage_base + (size_t)s * p.stage_bytes + (size_t)v * 16) = o;
        } else {
          uint16_t* dst = in_a ? row_a + (int64_t)v * 8 : row_b + (int64_t)(v - na) * 8;
          *reinterpret_cast<uint4*>(dst) = o;
        }
      }
    }
    if (kTmaStore) {
      fence_proxy_async_smem();  // make this thread's stage writes visible to the bulk copy
      __syncthreads();
      if (tid == 0) {
        uint8_t* st_out = stage_base + (size_t)s * p.stage_bytes;
        bulk_s2g(row_a, st_out, (uint32_t)na * 16u);
        if (rb >= 0) bulk_s2g(row_b, st_out + (size_t)na * 16, (uint32_t)(nv - na) * 16u);
        bulk_commit();
      }
    }
    // Masked columns and pitch padding: 16-byte zero stores, no loads.
    const int32_t za = pv - na;
    const int32_t zb = rb >= 0 ? pv - ((vb + 7) >> 3) : 0;
    const int32_t nb = (vb + 7) >> 3;
    for (int32_t zi = tid; zi < za + zb; zi += T) {
      uint16_t* dst = zi < za ? row_a + (int64_t)(na + zi) * 8 : row_b + (int64_t)(nb + zi - za) * 8;
      *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  }

  if (kTmaStore && tid == 0) bulk_wait_all();  // stores must finish reading shared memory

  // After a timeout: let this CTA's own copies in flight land (bounded)
  // before the shared memory they target is released.
  if (tid == 0 && k < n_mine) {
    for (int32_t r = k; r < n_issued; ++r)
      (void)mbar_wait_bounded(&full[r % S], (uint32_t)((r / S) & 1), g.timeout_ns);
  }
}

}  // namespace cs
