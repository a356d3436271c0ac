// Cluster-resident causal softmax for long rows (the `online` kernel choice,
// and the automatic one once a row pair no longer fits the row-resident
// kernel's shared memory).
//
// One row is spread over the C CTAs of a thread-block cluster (C = 2, 4 or
// 8), so that the row stays resident in the cluster's shared memory and HBM
// sees one read of its causal prefix and one write of the row:
//
//  * the row, padding included, is cut into blocks of B 16-byte vectors; CTA
//    r of the cluster owns blocks r, r + C, r + 2C, ... (dealt round-robin, so
//    every CTA holds an even share of every row, causal triangle included);
//  * a producer lane streams the CTA's blocks of each row into a ring of S
//    stages with 1-D TMA bulk copies (completing on a `full` mbarrier), writes
//    the CTA's masked blocks with bulk stores from a zeroed buffer, and sends
//    the normalised blocks from their stage with bulk stores before the
//    stage is refilled;
//  * consumer warps make three passes over the CTA's blocks in shared memory:
//    each warp's max, its sum of exp2((x - m_w) * scale*log2 e), and -- once
//    the row's statistics are known -- p = exp2((x - M) * scale*log2 e) / S;
//  * between passes 2 and 3 the CTAs exchange their (max, sum) partials
//    through distributed shared memory: consumer warp 0 merges the CTA's
//    warps, writes the CTA's partial into slot [stage][rank] of every CTA of
//    the cluster (st.shared::cluster) and arrives on that CTA's exchange
//    mbarrier (expected count C); every CTA waits on its own barrier and
//    merges the C partials. Slots and barriers are per stage: a CTA writes the
//    slot of row j + S only after it has received every CTA's partial of row
//    j + S - 1, which each CTA sends after reading the slot of row j.
//
// Every CTA loads its own blocks from global memory with plain bulk copies.
// Every wait is bounded (Geometry::timeout_ns) and reports kStatusTimeout; a
// CTA that gives up stops sending partials, so its peers' waits run out too.
// A cluster barrier after the barriers are initialised, and one before exit,
// keep every CTA's shared memory alive while its peers may access it.
#pragma once

#include "common.cuh"
#include "geometry.cuh"

namespace cs {

constexpr int kClusterMax = 16;        // CTAs per cluster (above 8: the non-portable opt-in)
constexpr int kClusterBlockVec = 128;  // vectors per block (2 KB)
constexpr int kClusterZeroBytes = kClusterBlockVec * 16;

struct ClusterParams {
  Geometry g;
  int64_t total_rows;   // batch * rows (flat rows)
  int32_t csize;        // C: CTAs per cluster
  int32_t stage_blocks; // blocks a CTA holds of one row (ceil(blocks per row / C))
  int32_t stages;       // S: ring depth (rows in flight per CTA)
};

// Shared memory after the stages: zero buffer, W (max, sum) warp partials per
// stage, C CTA partials per stage, full, empty and exchange mbarriers per
// stage, the row each stage holds (element offset, vectors) for the
// producer's stores, and the abort flag.
__host__ __device__ constexpr int cluster_tail_bytes(int stages) {
  return kClusterZeroBytes + stages * 32 * 8 + stages * kClusterMax * 8 + 3 * stages * 8 + stages * 16 + 16;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_f2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_parity_cluster(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Wait (bounded) for a phase completed by arrivals from other CTAs of the
// cluster, with cluster-scope acquire so their shared-memory stores are seen.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  if (mbar_try_wait_parity_cluster(bar, parity, 0u)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try_wait_parity_cluster(bar, parity, 200000u)) return true;
    if (global_timer_ns() - start > timeout_ns) return false;
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// (m, s) merge of online-softmax partials; m = -inf is an empty partial.
__device__ __forceinline__ void cluster_merge(float& m, float& s, float m2, float s2, float sl) {
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

__global__ void __launch_bounds__(544, 1) cluster_kernel(const __grid_constant__ ClusterParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Geometry& g = p.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = (blockDim.x >> 5) - 1;  // consumer warps; warp W is the producer
  const int S = p.stages;
  const int32_t C = p.csize;
  const uint32_t rank = cluster_rank();
  const size_t stage_bytes = (size_t)p.stage_blocks * kClusterBlockVec * 16;
  uint8_t* stage_base = smem;
  uint8_t* zero_buf = smem + (size_t)S * stage_bytes;
  float2* red = reinterpret_cast<float2*>(zero_buf + kClusterZeroBytes);  // [S][32]
  float2* xpart = red + S * 32;                                           // [S][kClusterMax]
  uint64_t* full = reinterpret_cast<uint64_t*>(xpart + S * kClusterMax);
  uint64_t* empty = full + S;
  uint64_t* xbar = empty + S;
  int64_t* held_off = reinterpret_cast<int64_t*>(xbar + S);      // [S] producer only
  int32_t* held_nvec = reinterpret_cast<int32_t*>(held_off + S);  // [S] producer only
  volatile int* abort_flag = reinterpret_cast<volatile int*>(held_off + 2 * S);

  const uint32_t nclusters = gridDim.x / (uint32_t)C;
  const uint32_t q = blockIdx.x / (uint32_t)C;  // this CTA's cluster; its rows are q + j*nclusters
  const bool skip_loads = (g.flags & kFlagSkipLoads) != 0;
  const int32_t pv = g.pitch >> 3;
  const int32_t nblk = (pv + kClusterBlockVec - 1) / kClusterBlockVec;  // blocks per padded row
  const float sl = g.scale * kLog2e;
  const float2 sl2 = make_float2(sl, sl);
  const bool zero_scale = sl == 0.f;

  for (int i = tid; i < kClusterZeroBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(zero_buf)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (uint32_t)W);
      mbar_init(&xbar[s], (uint32_t)C);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers exist before any peer arrives on them
  pdl_trigger();

  // This CTA's blocks of a row: local block t is row block rank + t*C; the
  // number of them, and the vectors of block t that hold causal data.
  const int32_t my_blocks = nblk > (int32_t)rank ? (nblk - 1 - (int32_t)rank) / C + 1 : 0;
  auto block_valid_vec = [&](int32_t t, int32_t nvec) {
    const int32_t v0 = ((int32_t)rank + t * C) * kClusterBlockVec;
    int32_t n = nvec - v0;
    n = n < 0 ? 0 : (n > kClusterBlockVec ? kClusterBlockVec : n);
    return n;
  };

  if (warp == W) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip_loads) {
      pdl_wait();  // inputs written, outputs read by the previous kernel: done
      auto store_row = [&](int s) {
        const uint8_t* st = stage_base + (size_t)s * stage_bytes;
        for (int32_t t = 0; t < my_blocks; ++t) {
          const int32_t n = block_valid_vec(t, held_nvec[s]);
          if (n == 0) break;
          bulk_s2g(g.out + held_off[s] + (int64_t)((int32_t)rank + t * C) * kClusterBlockVec * 8,
                   st + (size_t)t * kClusterBlockVec * 16, (uint32_t)n * 16u);
        }
        bulk_commit();
      };
      bool aborted = false;
      int64_t j = 0;   // rows issued
      RingPos pos;     // the stage of row j
      RowCursor cur(g, q, nclusters);
      for (; cur.inside(g); ++j, cur.next(g), pos.next(S)) {
        const int s = pos.s;
        if (j >= S) {
          // The stage's previous row: the phase before the current one.
          if (!mbar_wait_bounded(&empty[s], pos.ph ^ 1u, g.timeout_ns)) {
            aborted = true;
            *abort_flag = 1;
            if (g.status) atomicOr(g.status, kStatusTimeout);
            break;
          }
          if (*abort_flag) {  // the consumers gave up (a wait of this CTA or of a peer ran out)
            aborted = true;
            break;
          }
          store_row(s);
          bulk_wait_read_all();  // the stage is read out before it is refilled
        }
        const int64_t off = cur.offset(g);
        const int32_t nvec = (valid_cols(g, cur.i) + 7) >> 3;
        uint32_t bytes = 0;
        for (int32_t t = 0; t < my_blocks; ++t) bytes += (uint32_t)block_valid_vec(t, nvec) * 16u;
        mbar_arrive_expect_tx(&full[s], bytes);
        uint8_t* dst = stage_base + (size_t)s * stage_bytes;
        for (int32_t t = 0; t < my_blocks; ++t) {
          const int32_t n = block_valid_vec(t, nvec);
          const int64_t v0 = (int64_t)((int32_t)rank + t * C) * kClusterBlockVec;
          if (n > 0)
            bulk_g2s(dst + (size_t)t * kClusterBlockVec * 16, g.in + off + v0 * 8, (uint32_t)n * 16u, &full[s]);
          // Masked part of the block (and pitch padding): zeros.
          const int64_t z0 = v0 + n;
          const int64_t z1 = v0 + kClusterBlockVec < pv ? v0 + kClusterBlockVec : pv;
          if (z1 > z0) bulk_s2g(g.out + off + z0 * 8, zero_buf, (uint32_t)(z1 - z0) * 16u);
        }
        bulk_commit();
        bulk_wait_read_16();
        held_off[s] = off;
        held_nvec[s] = nvec;
      }
      if (!aborted) {
        // Outputs of the rows still held: the S stages from row j on hold
        // rows j - S .. j - 1 (those that exist), each released in the phase
        // before its position's.
        RingPos f = pos;
        for (int k = 0; k < S; ++k, f.next(S)) {
          if (j + k < S) continue;
          if (!mbar_wait_bounded(&empty[f.s], f.ph ^ 1u, g.timeout_ns)) {
            if (g.status) atomicOr(g.status, kStatusTimeout);
            break;
          }
          store_row(f.s);
        }
      }
      bulk_wait_all();
      // After an abort: the loads still in flight. Stage k's last row is
      // d = (pos.s - 1 - k) mod S rows back, in the current lap for
      // k < pos.s and in the previous one otherwise.
      if (aborted)
        for (int k = 0; k < S; ++k) {
          const int d = (pos.s - 1 - k + S) % S;
          if (j - 1 - d < 0) continue;
          (void)mbar_wait_bounded(&full[k], k < pos.s ? pos.ph : pos.ph ^ 1u, g.timeout_ns);
        }
    }
  } else {
    // ------------------------------------------------------------ consumers
    // (shared memory only: the producer makes every global access)
    const uint32_t xpart_local = smem_addr(xpart);
    const uint32_t xbar_local = smem_addr(xbar);
    int s = 0;
    uint32_t parity = 0;
    for (RowCursor cur(g, q, nclusters); cur.inside(g); cur.next(g)) {
      const int32_t valid = valid_cols(g, cur.i);
      const int32_t nvec = (valid + 7) >> 3;
      const bool ok = mbar_wait_bounded(&full[s], parity, g.timeout_ns);
      if (!ok) {
        *abort_flag = 1;
        if (g.status) atomicOr(g.status, kStatusTimeout);
      }
      const uint8_t* st = stage_base + (size_t)s * stage_bytes;
      constexpr uint32_t kNeg2 = kHalfNegInf | (kHalfNegInf << 16);
      // Warp w takes local blocks w, w + W, ...; lane l vectors l, l + 32, ... of each.
      auto load = [&](int32_t t, int32_t i) {
        uint4 r = *reinterpret_cast<const uint4*>(st + ((size_t)t * kClusterBlockVec + i) * 16);
        const int32_t v = ((int32_t)rank + t * C) * kClusterBlockVec + i;  // vector within the row
        const int32_t lim = valid - v * 8;
        if (lim < 8) r = mask_tail_neg_inf(r, lim);
        return r;
      };
      // Pass 1: the warp's max.
      uint32_t hm = kNeg2;
      if (ok)
        for (int32_t t = warp; t < my_blocks; t += W) {
          const int32_t n = block_valid_vec(t, nvec);
          for (int32_t i = lane; i < n; i += 32) {
            const uint4 r = load(t, i);
            hm = h2_bits(__hmax2(bits_h2(hm), __hmax2(__hmax2(bits_h2(r.x), bits_h2(r.y)),
                                                       __hmax2(bits_h2(r.z), bits_h2(r.w)))));
          }
        }
      const __half2 hm2 = bits_h2(hm);
      const float mw = redux_max(__half2float(__hmax(__low2half(hm2), __high2half(hm2))));
      // Pass 2: the warp's sum relative to its own max.
      float2 acc = make_float2(0.f, 0.f);
      if (ok && mw > -INFINITY) {
        const float2 nm2 = make_float2(-mw, -mw);
        for (int32_t t = warp; t < my_blocks; t += W) {
          const int32_t n = block_valid_vec(t, nvec);
          for (int32_t i = lane; i < n; i += 32) {
            const uint4 r = load(t, i);
            const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              float2 e;
              if (zero_scale) {
                e.x = (w4[qq] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
                e.y = (w4[qq] >> 16) == kHalfNegInf ? 0.f : 1.f;
              } else {
                const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w4[qq])), nm2), sl2);
                e = make_float2(ex2(d.x), ex2(d.y));
              }
              acc = __fadd2_rn(acc, e);
            }
          }
        }
      }
      const float sw = warp_sum(acc.x + acc.y);
      float2* rs = red + s * 32;
      if (lane == 0) rs[warp] = make_float2(mw, sw);
      // Consumer warps only; every warp learns whether any of them (or the
      // producer, through the flag) gave up, so they stop or go on together.
      bool stop = bar_red_or(1, W * 32, !ok || *abort_flag);
      if (warp == 0 && !stop) {
        // The CTA's partial, to slot [s][rank] of every CTA of the cluster.
        float2 ps = lane < W ? rs[lane] : make_float2(-INFINITY, 0.f);
        float m = ps.x, sm = ps.y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
          const float s2 = __shfl_xor_sync(0xffffffffu, sm, o);
          cluster_merge(m, sm, m2, s2, sl);
        }
        if (lane < C) {
          const uint32_t slot = xpart_local + (uint32_t)((s * kClusterMax + (int)rank) * 8);
          st_cluster_f2(map_to_rank(slot, (uint32_t)lane), m, sm);
          mbar_arrive_remote(map_to_rank(xbar_local + (uint32_t)(s * 8), (uint32_t)lane));
        }
        // Warp 0 waits for the C partials of the row (cluster-scope acquire);
        // the barrier below orders that before the other warps read them.
        if (!mbar_wait_cluster_bounded(&xbar[s], parity, g.timeout_ns)) {
          if (lane == 0) {
            *abort_flag = 1;
            if (g.status) atomicOr(g.status, kStatusTimeout);
          }
          stop = true;
        }
      }
      stop = bar_red_or(1, W * 32, stop);
      if (stop) {
        // Hand the stage back so the producer is not left waiting, then stop.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        break;
      }
      const float2 cp = lane < C ? xpart[s * kClusterMax + lane] : make_float2(-INFINITY, 0.f);
      float M = cp.x, Ssum = cp.y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, M, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, Ssum, o);
        cluster_merge(M, Ssum, m2, s2, sl);
      }
      const float rcp = rcp_rn(Ssum);
      const float2 r2 = make_float2(rcp, rcp);
      const float2 nM2 = make_float2(-M, -M);
      // Pass 3: normalise into the stage (the producer stores it).
      uint8_t* stw = stage_base + (size_t)s * stage_bytes;
      for (int32_t t = warp; t < my_blocks; t += W) {
        const int32_t n = block_valid_vec(t, nvec);
        for (int32_t i = lane; i < n; i += 32) {
          const uint4 r = load(t, i);
          const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
          uint32_t o[4];
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            float2 e;
            if (zero_scale) {
              e.x = (w4[qq] & 0xFFFFu) == kHalfNegInf ? 0.f : 1.f;
              e.y = (w4[qq] >> 16) == kHalfNegInf ? 0.f : 1.f;
            } else {
              const float2 d = __fmul2_rn(__fadd2_rn(__half22float2(bits_h2(w4[qq])), nM2), sl2);
              e = make_float2(ex2(d.x), ex2(d.y));
            }
            const float2 pr = __fmul2_rn(e, r2);
            o[qq] = float2_to_half2_bits(pr.x, pr.y);
          }
          *reinterpret_cast<uint4*>(stw + ((size_t)t * kClusterBlockVec + i) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_proxy_async_smem();  // outputs visible to the bulk-store engine
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == S) {
        s = 0;
        parity ^= 1u;
      }
    }
  }
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while a peer may still write its shared memory
}

}  // namespace cs
