// Narrow-row causal softmax (the `warp` kernel choice: cols <= 32 through the
// public selector; the same code serves rows of up to 256 columns).
//
// Replaces gpu/src/main.rs:164-198 (one warp per row, one 2-byte value per
// lane): here a row is owned by L = next_pow2(ceil(cols / 8)) lanes, each
// holding one 16-byte vector, so a warp covers 32 / L rows per step. Lanes
// whose vector lies wholly above the diagonal skip the load; max and sum are
// XOR butterflies confined to the L-lane group; each lane writes its vector
// (probabilities or zeros) and zero vectors at sub + L, sub + 2L, ... up to
// the pitch, so padding of any width is cleared.
#pragma once

#include "common.cuh"
#include "geometry.cuh"

namespace cs {

struct NarrowParams {
  Geometry g;
  int64_t total_rows;  // batch * rows
};

template <int L>
__global__ void __launch_bounds__(256) narrow_kernel(const __grid_constant__ NarrowParams p) {
  constexpr int R = 32 / L;  // rows per warp step
  const Geometry& g = p.g;
  const int lane = threadIdx.x & 31;
  const int sub = lane % L;  // this lane's vector within its row
  const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int32_t pv = g.pitch >> 3;
  const float sl = g.scale * kLog2e;
  pdl_trigger();
  pdl_wait();

  for (int64_t base = warp_id * R; base < p.total_rows; base += n_warps * R) {
    const int64_t flat = base + lane / L;
    const bool row_ok = flat < p.total_rows;
    const int64_t b = row_ok ? flat / g.rows : 0;
    const int32_t i = row_ok ? (int32_t)(flat - b * g.rows) : 0;
    const int32_t valid = row_ok ? valid_cols(g, i) : 0;
    const int32_t nvec = (valid + 7) >> 3;
    const int64_t off = b * g.batch_stride + (int64_t)i * g.pitch + (int64_t)sub * 8;

    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (row_ok && sub < nvec) raw = __ldg(reinterpret_cast<const uint4*>(g.in + off));
    const int32_t lim = valid - sub * 8;
    float z[8];
    {
      const float2 f0 = half2_bits_to_float2(raw.x), f1 = half2_bits_to_float2(raw.y);
      const float2 f2 = half2_bits_to_float2(raw.z), f3 = half2_bits_to_float2(raw.w);
      z[0] = f0.x; z[1] = f0.y; z[2] = f1.x; z[3] = f1.y;
      z[4] = f2.x; z[5] = f2.y; z[6] = f3.x; z[7] = f3.y;
    }
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < lim) m = fmaxf(m, z[e]);
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // exp2((x - max) * scale*log2(e)): exactly 1 for the maximum at any scale.
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      z[e] = e < lim ? ex2((z[e] - m) * sl) : 0.f;
      s += z[e];
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = rcp_rn(s);
    if (row_ok) {
      uint4 o;
      if (sub < nvec) {
        o.x = float2_to_half2_bits(z[0] * inv, z[1] * inv);
        o.y = float2_to_half2_bits(z[2] * inv, z[3] * inv);
        o.z = float2_to_half2_bits(z[4] * inv, z[5] * inv);
        o.w = float2_to_half2_bits(z[6] * inv, z[7] * inv);
      } else {
        o = make_uint4(0u, 0u, 0u, 0u);
      }
      if (sub < pv) *reinterpret_cast<uint4*>(g.out + off) = o;
      for (int32_t v = sub + L; v < pv; v += L)
        *reinterpret_cast<uint4*>(g.out + off + (int64_t)(v - sub) * 8) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

}  // namespace cs
