// Device-side helpers shared by the causal-softmax kernels (sm_100a).
//
// Hand-written PTX for the Blackwell async-copy path: mbarrier phase waits
// with a wall-clock bound, 1-D TMA bulk copies (cp.async.bulk) global->shared
// completing on an mbarrier transaction count, and the MUFU base-2
// exponential. Nothing here calls a CUDA math-library function.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace cs {

// Device status bit (written with atomicOr into the plan's status word); the
// other bits of the word are reserved and never set.
constexpr uint32_t kStatusTimeout = 1u;   // a bounded mbarrier wait ran out

// Debug flags a launch may carry (test-only code paths, off by default).
constexpr uint32_t kFlagSkipLoads = 1u;   // producer issues no copies: waits must time out

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch. The library launches its kernels with the
// programmatic-stream-serialization attribute, so a kernel's CTAs may start
// while the previous kernel in the stream is still running. pdl_wait blocks
// until that kernel has completed and its memory is visible (every kernel
// calls it before its first global load or store); pdl_trigger lets the next
// kernel's CTAs start their own set-up early. Both are no-ops for a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy) reads of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_parity(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `hint_ns` elapse, instead of re-issuing the probe.
__device__ __forceinline__ bool mbar_try_wait_parity_sleep(uint64_t* bar, uint32_t parity,
                                                           uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete, for at most
// `timeout_ns` of GPU wall time. Returns false when the bound ran out.
// Each probe suspends the thread (hint 0.2 ms) until the phase completes,
// so the loop neither spins hot nor steals issue slots from other warps.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t timeout_ns) {
  if (mbar_try_wait_parity(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_parity_sleep(bar, parity, 200000u)) return true;
    if (global_timer_ns() - start > timeout_ns) return false;
  }
}

// 1-D TMA bulk copy: `bytes` (multiple of 16) from global `src` (16-byte
// aligned) into shared `dst` (16-byte aligned); completion is signalled as
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Same, with an L2 eviction-priority hint (the score matrix is read once).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk prefetch of `bytes` (multiple of 16) at global `src` (16-byte aligned)
// into L2; no data reaches the SM and nothing completes on a barrier.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 1-D TMA bulk store shared -> global, tracked by the bulk async-group.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until all committed bulk stores have finished READING shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Bound the number of bulk-store groups in flight (their source reads).
__device__ __forceinline__ void bulk_wait_read_16() {
  asm volatile("cp.async.bulk.wait_group.read 16;" ::: "memory");
}

// Wait until all committed bulk stores are complete (visible in global).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Barrier among the first `nthreads` threads (named barrier `id`) that also
// ORs a predicate over them: every participant gets the same answer.
__device__ __forceinline__ bool bar_red_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// A position in a ring of S stages: the stage and the parity of its current
// mbarrier phase, advanced one use at a time (no division by the depth).
struct RingPos {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next(int S) {
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
  }
};

// MUFU base-2 exponential (PTX ex2.approx; subnormal results flush to zero,
// which cannot change an FP16 probability: p <= e and e < 2^-126 rounds to 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Correctly rounded reciprocal (PTX rcp.rn): with e == 1 (zero scale) the
// probability is exactly RN(1/valid), as in the f32 specification.
__device__ __forceinline__ float rcp_rn(float x) {
  float y;
  asm("rcp.rn.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t bits) {
  __half2 h = *reinterpret_cast<__half2*>(&bits);
  return __half22float2(h);
}

__device__ __forceinline__ uint32_t float2_to_half2_bits(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Packed-half helpers for the max pass (comparisons of halves are exact).
constexpr uint32_t kHalfNegInf = 0xFC00u;

// Replace halves at element index >= lim (0..7 within a 16-byte vector)
// by -inf so they cannot win the row maximum.
__device__ __forceinline__ uint4 mask_tail_neg_inf(uint4 r, int32_t lim) {
  uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (2 * q >= lim) w[q] = (w[q] & 0xFFFF0000u) | kHalfNegInf;
    if (2 * q + 1 >= lim) w[q] = (w[q] & 0x0000FFFFu) | (kHalfNegInf << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ __half2 bits_h2(uint32_t b) { return *reinterpret_cast<__half2*>(&b); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Maximum of the 8 halves of a vector, as a half.
__device__ __forceinline__ __half max8_half(uint4 r) {
  const __half2 m = __hmax2(__hmax2(bits_h2(r.x), bits_h2(r.y)), __hmax2(bits_h2(r.z), bits_h2(r.w)));
  return __hmax(__low2half(m), __high2half(m));
}

// Butterfly max of a packed half pair across the warp.
__device__ __forceinline__ uint32_t warp_max_h2(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v = h2_bits(__hmax2(bits_h2(v), bits_h2(__shfl_xor_sync(0xffffffffu, v, o))));
  return v;
}

// Single-instruction warp reductions (sm_100a redux.sync).
__device__ __forceinline__ float redux_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ uint32_t redux_add(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.add.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

// Warp sum of non-negative x <= 2^31 / 2^kShift, in fixed point with kShift
// fractional bits: each lane is rounded to 2^-(kShift+1), split into two
// 16-bit halves whose sums cannot overflow, and reduced with two integer
// redux instructions. Integers (zero-scale counts) are summed exactly.
template <int kShift>
__device__ __forceinline__ float warp_sum_fixed(float x) {
  const uint32_t q = __float2uint_rn(x * (float)(1u << kShift));
  const uint32_t hi = redux_add(q >> 16), lo = redux_add(q & 0xFFFFu);
  return ((float)hi * 65536.f + (float)lo) * (1.f / (float)(1u << kShift));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float2 warp_max2(float2 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x = fmaxf(v.x, __shfl_xor_sync(0xffffffffu, v.x, o));
    v.y = fmaxf(v.y, __shfl_xor_sync(0xffffffffu, v.y, o));
  }
  return v;
}

__device__ __forceinline__ float2 warp_sum2(float2 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  return v;
}

}  // namespace cs
