// Control kernel (the `baseline` kernel choice): plain global memory, no TMA,
// no shared-memory staging.
//
// Like gpu/src/main.rs:70-160 it gives each row one CTA and makes three
// passes over the causal prefix (max, sum, normalise), with a two-level
// reduction (warp butterfly, then the per-warp partials); unlike it, the
// passes use 16-byte vector loads, only the prefix is read, and the masked
// columns are written as 16-byte zero stores. It exists as a simple,
// independently written check on the faster kernels, not for speed.
#pragma once

#include "common.cuh"
#include "geometry.cuh"

namespace cs {

struct BaselineParams {
  Geometry g;
  int64_t total_rows;
};

__device__ __forceinline__ void load8(const uint16_t* src, float z[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
  const float2 f0 = half2_bits_to_float2(raw.x), f1 = half2_bits_to_float2(raw.y);
  const float2 f2 = half2_bits_to_float2(raw.z), f3 = half2_bits_to_float2(raw.w);
  z[0] = f0.x; z[1] = f0.y; z[2] = f1.x; z[3] = f1.y;
  z[4] = f2.x; z[5] = f2.y; z[6] = f3.x; z[7] = f3.y;
}

// Block-wide reduction of one float (max or sum); every thread gets the result.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  v = kMax ? warp_max(v) : warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : (kMax ? -INFINITY : 0.f);
  t = kMax ? warp_max(t) : warp_sum(t);
  __syncthreads();  // red[] may be rewritten by the next reduction
  return t;
}

__global__ void __launch_bounds__(256) baseline_kernel(const __grid_constant__ BaselineParams p) {
  __shared__ float red[32];
  const Geometry& g = p.g;
  const int32_t pv = g.pitch >> 3;
  const float sl = g.scale * kLog2e;  // exponents (x - max) * scale*log2(e)
  pdl_trigger();
  pdl_wait();
  for (int64_t flat = blockIdx.x; flat < p.total_rows; flat += gridDim.x) {
    const int64_t b = flat / g.rows;
    const int32_t i = (int32_t)(flat - b * g.rows);
    const int32_t valid = valid_cols(g, i);
    const int32_t nvec = (valid + 7) >> 3;
    const int64_t off = b * g.batch_stride + (int64_t)i * g.pitch;
    const uint16_t* src = g.in + off;
    uint16_t* dst = g.out + off;

    float m = -INFINITY;
    for (int32_t v = threadIdx.x; v < nvec; v += blockDim.x) {
      float z[8];
      load8(src + (int64_t)v * 8, z);
      const int32_t lim = valid - v * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < lim) m = fmaxf(m, z[e]);
    }
    m = block_reduce<true>(m, red);

    float s = 0.f;
    for (int32_t v = threadIdx.x; v < nvec; v += blockDim.x) {
      float z[8];
      load8(src + (int64_t)v * 8, z);
      const int32_t lim = valid - v * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) s += e < lim ? ex2((z[e] - m) * sl) : 0.f;
    }
    s = block_reduce<false>(s, red);
    const float inv = rcp_rn(s);

    for (int32_t v = threadIdx.x; v < pv; v += blockDim.x) {
      uint4 o = make_uint4(0u, 0u, 0u, 0u);
      if (v < nvec) {
        float z[8];
        load8(src + (int64_t)v * 8, z);
        const int32_t lim = valid - v * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) z[e] = e < lim ? ex2((z[e] - m) * sl) * inv : 0.f;
        o.x = float2_to_half2_bits(z[0], z[1]);
        o.y = float2_to_half2_bits(z[2], z[3]);
        o.z = float2_to_half2_bits(z[4], z[5]);
        o.w = float2_to_half2_bits(z[6], z[7]);
      }
      *reinterpret_cast<uint4*>(dst + (int64_t)v * 8) = o;
    }
  }
}

}  // namespace cs
