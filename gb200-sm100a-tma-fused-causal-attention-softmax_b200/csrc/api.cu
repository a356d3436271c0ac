// C ABI of the B200 fused causal softmax: argument checks, kernel selection,
// launch geometry, plans, one-shot launches and host-buffer sessions.
//
// This file replaces the reference's typed dispatch boundary
// (gpu/src/driver.rs:12-233) and its TMA descriptor setup
// (gpu/src/main.rs:730-774). Kernels come from kernels/*.cuh.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>
#if defined(__x86_64__)
#include <emmintrin.h>
#endif

#include "causal_softmax.h"
#include "kernels/baseline.cuh"
#include "kernels/cluster.cuh"
#include "kernels/narrow.cuh"
#include "kernels/online.cuh"
#include "kernels/rowres.cuh"
#include "kernels/util.cuh"

namespace {

using cs::Geometry;

constexpr int kMaxDevices = 64;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s of GPU time per wait
constexpr int kDefaultStages = 3;
constexpr int64_t kRingBytesPerSm = 72 * 1024;  // row-resident ring bytes per SM (target)
constexpr int kMaxAutoStages = 8;
constexpr int kOnlineDefaultStages = 8;
constexpr int kMaxStages = 32;  // ring depth a tuning request may ask for (shared memory decides the rest)
constexpr int64_t kI32Max = 2147483647;
constexpr int64_t kMaxUnitsPerLaunch = int64_t(1) << 30;  // row-resident kernel, 32-bit unit index

thread_local char t_detail[256];

int cuda_fail(cudaError_t e, const char* what) {
  std::snprintf(t_detail, sizeof t_detail, "%s: %s", what, cudaGetErrorString(e));
  return CS_ERR_CUDA;
}

#define CS_CUDA(call)                                 \
  do {                                                \
    cudaError_t _e = (call);                          \
    if (_e != cudaSuccess) return cuda_fail(_e, #call); \
  } while (0)

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int major = 0, minor = 0;
  int max_smem_optin = 0;
  uint32_t* oneshot_status = nullptr;  // status word for cs_softmax*
  uint32_t* noalloc_status = nullptr;  // device address of g_noalloc_status
  int row_regs[2][16] = {};            // registers per thread of each row-resident variant
  bool attrs_set = false;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
    if (prev_ != dev) ok_ = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev_ >= 0 && ok_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = -1;
  bool ok_ = true;
};

// Instantiations of the row-resident kernel (index, V vectors per consumer
// lane, launch bounds MAXT threads / MINB resident CTAs per SM, which set the
// register budget). The planner picks among them by occupancy and register
// budget (rowres_pick).
#define CS_ROW_VARIANTS(X) \
  X(0, 8, 256, 1)          \
  X(1, 8, 448, 1)          \
  X(2, 4, 512, 1)          \
  X(3, 2, 1024, 1)         \
  X(4, 4, 224, 4)          \
  X(5, 2, 352, 3)          \
  X(6, 4, 384, 2)          \
  X(7, 0, 1024, 1)

struct RowVariant {
  int vec;
  int maxt;
  int minb;
};
#define CS_ROW_ENTRY(i, v, t, b) {v, t, b},
constexpr RowVariant kRowVariants[] = {CS_ROW_VARIANTS(CS_ROW_ENTRY)};
#undef CS_ROW_ENTRY
constexpr int kNumRowVariants = (int)(sizeof(kRowVariants) / sizeof(kRowVariants[0]));

void* rowres_kernel_ptr(int variant, bool ts) {
  switch (variant) {
#define CS_ROW_PTR(i, v, t, b)                                                          \
  case i:                                                                               \
    return ts ? reinterpret_cast<void*>(&cs::rowres_kernel<v, t, b, true>)              \
              : reinterpret_cast<void*>(&cs::rowres_kernel<v, t, b, false>);
    CS_ROW_VARIANTS(CS_ROW_PTR)
#undef CS_ROW_PTR
    default: return nullptr;
  }
}

// Per-device properties and one-time kernel attributes (max dynamic smem).
int device_info(int dev, DeviceInfo** out) {
  if (dev < 0 || dev >= kMaxDevices) return CS_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || dev >= n) {
      std::snprintf(t_detail, sizeof t_detail, "device %d not present (%d devices)", dev, n);
      return CS_ERR_DEVICE;
    }
    CS_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    CS_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
    CS_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
    CS_CUDA(cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (d.major != 10) {
      std::snprintf(t_detail, sizeof t_detail, "sm_100a build needs compute capability 10.x, found %d.%d",
                    d.major, d.minor);
      return CS_ERR_DEVICE;
    }
    d.ready = true;
  }
  if (!d.attrs_set) {
    DeviceGuard guard(dev);
    if (!guard.ok()) return CS_ERR_DEVICE;
    for (int ts = 0; ts < 2; ++ts)
      for (int v = 0; v < kNumRowVariants; ++v) {
        CS_CUDA(cudaFuncSetAttribute(rowres_kernel_ptr(v, ts != 0),
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem_optin));
        cudaFuncAttributes fa{};
        CS_CUDA(cudaFuncGetAttributes(&fa, rowres_kernel_ptr(v, ts != 0)));
        d.row_regs[ts][v] = fa.numRegs;
      }
    CS_CUDA(cudaFuncSetAttribute(reinterpret_cast<void*>(&cs::online_kernel<1>),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem_optin));
    CS_CUDA(cudaFuncSetAttribute(reinterpret_cast<void*>(&cs::online_kernel<2>),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem_optin));
    CS_CUDA(cudaFuncSetAttribute(reinterpret_cast<void*>(&cs::cluster_kernel),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem_optin));
    CS_CUDA(cudaFuncSetAttribute(reinterpret_cast<void*>(&cs::cluster_kernel),
                                 cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    // Every other kernel a launch may pick, so that the driver has all of the
    // library's code in place once this set-up is done (it may take device
    // memory for it); later launches then add nothing on the device.
    const void* others[] = {reinterpret_cast<const void*>(&cs::narrow_kernel<1>),
                            reinterpret_cast<const void*>(&cs::narrow_kernel<2>),
                            reinterpret_cast<const void*>(&cs::narrow_kernel<4>),
                            reinterpret_cast<const void*>(&cs::narrow_kernel<8>),
                            reinterpret_cast<const void*>(&cs::narrow_kernel<16>),
                            reinterpret_cast<const void*>(&cs::narrow_kernel<32>),
                            reinterpret_cast<const void*>(&cs::baseline_kernel)};
    for (const void* k : others) {
      cudaFuncAttributes fa{};
      CS_CUDA(cudaFuncGetAttributes(&fa, k));
    }
    d.attrs_set = true;
  }
  *out = &d;
  return CS_OK;
}

int64_t padded_pitch(int64_t cols) { return (cols + 7) & ~int64_t(7); }

bool is_known_kernel(int k) { return k >= CS_KERNEL_AUTO && k <= CS_KERNEL_ONLINE; }

// Causal element count of rows [row_offset, row_offset + rows).
double causal_elements(int64_t rows, int64_t cols, int64_t row_offset) {
  int64_t tri = cols - 1 - row_offset;
  if (tri < 0) tri = 0;
  if (tri > rows) tri = rows;
  const double t = (double)tri;
  return t * (double)(row_offset + 1) + t * (t - 1.0) / 2.0 + (double)(rows - tri) * (double)cols;
}

// Causal element count of a launch's rows (both row blocks of a folded one),
// with rows clipped to `cols` columns.
double geometry_causal_elements(const Geometry& g, int64_t cols) {
  const double first = g.split_row > 0 ? causal_elements(g.split_row, cols, g.row_offset) : 0.0;
  return first + causal_elements((int64_t)g.rows - g.split_row, cols,
                                 (int64_t)g.row_offset + g.split_row + g.split_shift);
}

int validate_args(int64_t batch, int64_t batch_stride, int64_t rows, int64_t cols, int64_t pitch,
                  int64_t row_offset, float scale) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return CS_ERR_EMPTY;
  if (rows > kI32Max || cols > kI32Max || row_offset < 0 || row_offset > kI32Max - rows)
    return CS_ERR_WRONG_LENGTH;
  if (pitch < cols || (pitch & 7) != 0 || pitch > kI32Max) return CS_ERR_PITCH;
  if (!std::isfinite(scale) || !(scale >= 0.0f && scale <= CS_MAX_SCALE)) return CS_ERR_BAD_SCALE;
  const int64_t mat = rows * pitch;  // < 2^62
  if (batch > 1) {
    if (batch_stride < mat || (batch_stride & 7) != 0) return CS_ERR_WRONG_LENGTH;
    if (batch - 1 > (INT64_MAX - mat) / batch_stride) return CS_ERR_WRONG_LENGTH;
  }
  return CS_OK;
}

// ---------------------------------------------------------------------------
// Launch planning
// ---------------------------------------------------------------------------

struct Tuning {
  int vec = 0;         // 0: automatic
  int stages = 0;      // 0: automatic
  int hint = -1;       // -1: automatic
  int zero_tma = -1;   // -1: automatic
  int prefetch = -1;   // row-resident: units per CTA prefetched into L2 before the PDL wait; -1 automatic
};

// Units per CTA whose input rows the row-resident kernel pulls into L2
// while the previous kernel in the stream finishes (the first ring stages'
// are always prefetched). Measured on B200, back-to-back launches on the
// same GPU against 2: 8192^2 -0.8% time with 4, +2.5% with 8, +7% with 16;
// 4096^2 and batched 4096^2 level.
constexpr int kDefaultPrefetch = 4;

struct LaunchPlan {
  int kernel = 0;
  int grid = 0, block = 0, smem = 0, stages = 0, vec = 0, variant = 0, ctas_per_sm = 0;
  bool dyn_sched = false;  // row-resident kernel claims units through g.sched
  int64_t units = 0;
  int narrow_lanes = 0;
  cs::RowResParams rr{};
  cs::OnlineParams on{};
  bool cluster = false;    // online: the cluster-resident kernel (cl) instead of on
  cs::ClusterParams cl{};
  cs::NarrowParams nr{};
  cs::BaselineParams bl{};
};

int64_t rowres_max_vectors(const Geometry& g, const cs::UnitMap& m) { return cs::unit_max_vectors(g, m); }

// CTA size of variant i for units of up to max_nv vectors: each consumer
// warp owns 32*V vectors of one row, a row pair needs one warp more than its
// total in the worst split, and one producer warp is added. False if the
// variant cannot hold such a unit.
bool rowres_block(int64_t max_nv, bool paired, int i, int* block) {
  const int v = kRowVariants[i].vec;
  if (v == 0) {
    // Shared-memory passes: about 4 vectors per lane and pass, 2..31 consumer warps.
    const int64_t want = (max_nv + 127) / 128;
    const int64_t w = want < 2 ? 2 : (want > 31 ? 31 : want);
    *block = (int)(32 * (w + 1));
    return true;
  }
  const int64_t warps = (max_nv + 32 * v - 1) / (32 * v) + (paired ? 1 : 0) + 1;
  if (warps > 31 || 32 * warps > kRowVariants[i].maxt) return false;
  *block = (int)(32 * warps);
  return true;
}

// Whether tuning vec `want_vec` admits variant i (0: any; 2, 4, 8: that V;
// 16 + j: variant j only).
bool rowres_wanted(int want_vec, int i) {
  if (want_vec >= 16) return want_vec - 16 == i;
  return !want_vec || kRowVariants[i].vec == want_vec;
}

// Host-only fit test (no device queries): some admitted variant holds the unit.
bool rowres_shape(int64_t max_nv, bool paired, int want_vec) {
  int block = 0;
  for (int i = 0; i < kNumRowVariants; ++i)
    if (rowres_wanted(want_vec, i) && rowres_block(max_nv, paired, i, &block)) return true;
  return false;
}

// Variant groups in order of preference: V = 4 first, then the
// shared-memory passes (V = 0), then V = 8 and V = 2, which only a tuning
// request reaches. Measured on B200 over square widths 1024..32768: V = 4
// wins wherever it fits for single matrices (up to ~12000 columns: 4096^2
// 12.3 against 16.0 us, 8192^2 36.2 against 37.4 us, 12288^2 76.5 against
// 79.8 us); beyond, V = 0 beats V = 8 by 7-36% (16384^2: 5509 against 4655
// GB/s; 32768^2: 526 against 714 us). In steady state (many units per CTA,
// see kSteadyUnitsPerCta) V = 0 keeps more CTAs resident and wins instead,
// except near 4096 columns, where four V = 4 CTAs fill an SM: batched
// launches of ~2 GB, V = 0 against V = 4, GB/s: 2048 cols 4889/4381, 3072
// 5613/5327, 4096 5698/5827, 5120 5957/5847, 6144 6448/6108, 7168 6422/5830,
// 8192 6528/6013, 10240 6499/5464, 12288 6106/6191.
constexpr int kRowGroups[4][3] = {{4, 6, 2}, {7, -1, -1}, {0, 1, -1}, {5, 3, -1}};
constexpr int64_t kSteadyUnitsPerCta = 32;
// Widest units (16-byte vectors) of the band where V = 4 stays ahead in
// steady state: rows of ~3600 to ~4600 columns.
constexpr int64_t kV4BandLo = 450, kV4BandHi = 578;

// Pick the variant for units of up to max_nv vectors. Within a group the
// score is resident warps per SM x registers^1.5: more resident warps hide
// the per-unit latency, but a variant with a smaller register budget (and
// spills) must buy about 30% more warps to win (measured: 2048-wide rows run
// 7% faster on 4 CTAs x 87 registers than on 5 CTAs x 72).
int rowres_pick(const DeviceInfo& d, int64_t max_nv, bool paired, int want_vec, int stage_bytes,
                bool tma_store, int* variant, int* block) {
  for (const auto& group : kRowGroups) {
    double best = -1.0;
    for (int i : group) {
      int b = 0;
      if (i < 0 || !rowres_wanted(want_vec, i) || !rowres_block(max_nv, paired, i, &b)) continue;
      int per_sm = 0;
      CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rowres_kernel_ptr(i, tma_store), b,
                                                            2 * stage_bytes + cs::rowres_tail_bytes(2)));
      const double regs = d.row_regs[tma_store ? 1 : 0][i];
      const double score = (double)per_sm * (b / 32) * regs * std::sqrt(regs);
      if (per_sm > 0 && score > best) {
        best = score;
        *variant = i;
        *block = b;
      }
    }
    if (best > 0) return CS_OK;
  }
  return CS_ERR_UNSUPPORTED;
}

// Row-resident kernel geometry; CS_ERR_UNSUPPORTED when a unit does not fit.
int plan_rowres(const DeviceInfo& d, const Geometry& g, const Tuning& t, bool tma_store,
                LaunchPlan* lp) {
  cs::UnitMap m{};
  int64_t max_nv = 0;
  int variant = -1, block = 0, stage_bytes = 0;
  // Row pairs first; a pair may not fit where a single row still does.
  for (bool paired : {true, false}) {
    m = cs::make_unit_map(g, paired);
    max_nv = rowres_max_vectors(g, m);
    stage_bytes = (int)((max_nv * 16 + 127) / 128 * 128);
    const int rc = rowres_pick(d, max_nv, m.n_pairs > 0, t.vec, stage_bytes, tma_store, &variant, &block);
    if (rc == CS_OK) break;
    if (rc != CS_ERR_UNSUPPORTED) return rc;
  }
  if (variant >= 0 && t.vec == 0 && kRowVariants[variant].vec != 0 && (max_nv < kV4BandLo || max_nv > kV4BandHi)) {
    // Steady state: the shared-memory variant, if every CTA of its grid gets
    // at least kSteadyUnitsPerCta units.
    int v0 = -1, b0 = 0;
    if (rowres_pick(d, max_nv, m.n_pairs > 0, 16 + 7, stage_bytes, tma_store, &v0, &b0) == CS_OK) {
      int per_sm0 = 0;
      CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm0, rowres_kernel_ptr(v0, tma_store), b0,
                                                            2 * stage_bytes + cs::rowres_tail_bytes(2)));
      if (per_sm0 > 0 && m.total_units >= kSteadyUnitsPerCta * (int64_t)d.sms * per_sm0) {
        variant = v0;
        block = b0;
      }
    }
  }
  const int vec = variant >= 0 ? kRowVariants[variant].vec : 0;
  if (variant < 0) {
    std::snprintf(t_detail, sizeof t_detail, "row-resident kernel: %lld vectors per unit do not fit",
                  (long long)max_nv);
    return CS_ERR_UNSUPPORTED;
  }
  int stages = t.stages ? t.stages : kDefaultStages;
  if (!t.stages && vec == 0) {
    // Shared-memory passes: two stages (measured best or within 4% from
    // 4096 to 32768 columns; a third costs 10% at 32768^2).
    stages = 2;
  } else if (!t.stages) {
    // The ring depth that puts closest to kRingBytesPerSm of stages on each
    // SM (all its resident CTAs together), at least two, without losing a
    // resident CTA. Measured on B200 over square widths 2048..32768: 64-80 KB
    // per SM is best; a deeper ring costs up to 48% (32768^2 at 192 KB), a
    // shallower one up to 12%.
    double best = 1e30;
    int per_sm2 = 0;
    for (int s = 2; s <= kMaxAutoStages; ++s) {
      const int64_t sm = (int64_t)s * stage_bytes + cs::rowres_tail_bytes(s);
      if (sm > d.max_smem_optin) break;
      int per_sm = 0;
      CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rowres_kernel_ptr(variant, tma_store),
                                                            block, (size_t)sm));
      if (s == 2) per_sm2 = per_sm;
      if (per_sm < 1 || per_sm < per_sm2) break;
      const double dist = std::fabs(std::log((double)per_sm * s * stage_bytes / (double)kRingBytesPerSm));
      if (dist < best - 1e-9) {
        best = dist;
        stages = s;
      }
    }
    // A launch that gives each CTA fewer than kSteadyUnitsPerCta units is
    // shaped by its ramp: one stage more puts a deeper first batch of copies
    // in flight, where it keeps the resident CTAs (measured on B200, one
    // launch each: 4096^2 +1.8%, 6144^2 +6.6%, 8192^2 +4%, 4 x 4096^2 +4%,
    // 16 x 2048^2 +1.4%; at 55 units per CTA, 16 x 4096^2 and 4 x 8192^2, it
    // costs 1-3%).
    const int64_t sm_next = (int64_t)(stages + 1) * stage_bytes + cs::rowres_tail_bytes(stages + 1);
    if (stages < kMaxAutoStages && sm_next <= d.max_smem_optin) {
      int per_cur = 0, per_next = 0;
      CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &per_cur, rowres_kernel_ptr(variant, tma_store), block,
          (size_t)((int64_t)stages * stage_bytes + cs::rowres_tail_bytes(stages))));
      if (per_cur > 0 && m.total_units < kSteadyUnitsPerCta * (int64_t)d.sms * per_cur) {
        CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_next, rowres_kernel_ptr(variant, tma_store),
                                                              block, (size_t)sm_next));
        if (per_next >= per_cur) ++stages;
      }
    }
  }
  while (stages > 1 && (int64_t)stages * stage_bytes + cs::rowres_tail_bytes(stages) > d.max_smem_optin)
    --stages;
  const int smem = stages * stage_bytes + cs::rowres_tail_bytes(stages);
  // The bulk-store variant refills a stage one unit late, so it needs two.
  if (smem > d.max_smem_optin || ((!t.stages || tma_store) && stages < 2)) {
    std::snprintf(t_detail, sizeof t_detail, "row-resident kernel: stage of %d bytes too large", stage_bytes);
    return CS_ERR_UNSUPPORTED;
  }
  int per_sm = 0;
  CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rowres_kernel_ptr(variant, tma_store),
                                                        block, smem));
  if (per_sm < 1) {
    std::snprintf(t_detail, sizeof t_detail, "row-resident kernel: no resident CTA (block %d, smem %d)",
                  block, smem);
    return CS_ERR_UNSUPPORTED;
  }
  lp->kernel = tma_store ? CS_KERNEL_PIPELINE : CS_KERNEL_TMA;
  lp->units = m.total_units;
  lp->grid = (int)std::min<int64_t>(m.total_units, (int64_t)d.sms * per_sm);
  lp->block = block;
  lp->smem = smem;
  lp->stages = stages;
  lp->vec = vec;
  lp->variant = variant;
  lp->ctas_per_sm = per_sm;
  // Dynamic unit claiming for the shared-memory consumers only. Measured on
  // B200 against the static schedule on the same GPU: 32768^2 +3.2%,
  // 16384^2 +10%, 24576^2 -5%. The register-resident consumers compute each
  // unit's geometry before its data arrives, which needs the static
  // schedule; giving them the claiming producer cost 1.5-5%, and claiming
  // only each CTA's last units (whole, or one row at a time) cost 0.5-10%
  // on 4096^2 and 8192^2 single matrices.
  lp->dyn_sched = vec == 0;
  lp->rr.g = g;
  if (!lp->dyn_sched) lp->rr.g.sched = nullptr;
  lp->rr.m = m;
  lp->rr.stages = stages;
  lp->rr.stage_bytes = stage_bytes;
  // Measured on B200: the evict-first hint on the input copies costs ~3%.
  lp->rr.l2_hint = t.hint < 0 ? 0 : t.hint;
  lp->rr.zero_tma = t.zero_tma < 0 ? 1 : t.zero_tma;
  lp->rr.prefetch = t.prefetch < 0 ? kDefaultPrefetch : t.prefetch;
  return CS_OK;
}

// Online kernel launch shapes: 256 threads x 2 vectors (8 KB tiles), the
// automatic choice, or -- by tuning request (vec 1) -- 1024 threads x 1
// vector (16 KB tiles), which holds rows of up to ~114K columns resident on
// one CTA per SM. Measured on B200 (GB/s): 100000-column rows 2539 for the
// wide shape against 2858 for two fetches on four 256-thread CTAs per SM,
// 70000 columns 2430 against 3154, 32768^2 2348 against 3794 resident on
// three CTAs per SM: one resident row per SM leaves a bubble at every row
// boundary that several CTAs per SM hide.
// Cluster-resident online kernel: a row's blocks of 2 KB are dealt over the
// C CTAs of a cluster, so each CTA holds stage_blocks blocks of a row per
// stage. C is the smallest of 2, 4, 8 that keeps a stage within 24 blocks
// (48 KB), so that two stages of a few CTAs fit an SM; rows needing more are
// not served (CS_ERR_UNSUPPORTED).
int plan_cluster(const DeviceInfo& d, const Geometry& g, const Tuning& t, LaunchPlan* lp) {
  const int64_t pv = g.pitch / 8;
  const int64_t nblk = (pv + cs::kClusterBlockVec - 1) / cs::kClusterBlockVec;
  int csize = 0;
  int64_t stage_blocks = 0;
  for (int c : {2, 4, 8, 16}) {
    stage_blocks = (nblk + c - 1) / c;
    if (stage_blocks <= 24) {
      csize = c;
      break;
    }
  }
  if (!csize) {
    std::snprintf(t_detail, sizeof t_detail, "cluster kernel: rows of %lld vectors exceed 16 CTAs x 24 blocks",
                  (long long)pv);
    return CS_ERR_UNSUPPORTED;
  }
  const int stages = t.stages ? std::max(2, std::min(t.stages, 8)) : 2;
  const int warps = (int)std::max<int64_t>(2, std::min<int64_t>(16, stage_blocks));
  const int block = 32 * (warps + 1);
  const int smem = (int)(stages * stage_blocks * cs::kClusterBlockVec * 16) + cs::cluster_tail_bytes(stages);
  if (smem > d.max_smem_optin) return CS_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(csize * d.sms));
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_clusters = 0;
  CS_CUDA(cudaOccupancyMaxActiveClusters(&max_clusters, reinterpret_cast<void*>(&cs::cluster_kernel), &cfg));
  if (max_clusters < 1) return CS_ERR_UNSUPPORTED;
  const int64_t total_rows = g.batch * g.rows;
  lp->kernel = CS_KERNEL_ONLINE;
  lp->cluster = true;
  lp->units = total_rows;
  lp->grid = (int)(std::min<int64_t>(total_rows, max_clusters) * csize);
  lp->block = block;
  lp->smem = smem;
  lp->stages = stages;
  lp->vec = 3;
  lp->ctas_per_sm = (int)std::max<int64_t>(1, (int64_t)max_clusters * csize / d.sms);
  lp->cl.g = g;
  lp->cl.total_rows = total_rows;
  lp->cl.csize = csize;
  lp->cl.stage_blocks = (int32_t)stage_blocks;
  lp->cl.stages = stages;
  return CS_OK;
}

int plan_online(const DeviceInfo& d, const Geometry& g, const Tuning& t, LaunchPlan* lp) {
  if (t.vec == 3) return plan_cluster(d, g, t, lp);
  const int64_t widest = std::min<int64_t>(cs::abs_row(g, g.rows - 1) + 1, g.cols);
  const int64_t widest_vec = (widest + 7) / 8;
  auto max_stages_for = [&](int64_t tile_bytes) {
    return (int)std::min<int64_t>(kMaxStages, (d.max_smem_optin - cs::online_tail_bytes(kMaxStages)) / tile_bytes);
  };
  // Automatic shape, by the widest row (measured on B200, GB/s):
  //  * at most two default tiles: the short shape, six CTAs per SM
  //    (64 x 4096^2: 4395 against 3161 for the default shape);
  //  * up to the default ring (8 tiles, 32768 columns): the default shape,
  //    three CTAs per SM (32768^2 forced: 5452 against 4828 for the wide);
  //  * longer rows: the wide shape, one CTA per SM with the deepest ring
  //    that fits (13 stages of 15.5 KB hold rows of up to ~111K columns
  //    resident): 65536 / 70000 / 98304 / 100000 / 131072 columns 4685 /
  //    5043 / 5030 / 5080 / 4687 against 4432 / 4558 / 4137 / 4116 / 4002
  //    for the default shape on 4 stages (two fetches, 4 CTAs per SM).
  const bool short_rows = t.vec == 0 && widest_vec <= 2 * (int64_t)cs::kOnlineTileVec;
  const bool long_rows = t.vec == 0 && widest_vec > (int64_t)kOnlineDefaultStages * cs::kOnlineTileVec;
  const int vpt = (t.vec == 1 || long_rows) ? 1 : 2;
  const int threads = vpt == 1 ? cs::kOnlineWideThreads : short_rows ? cs::kOnlineShortThreads : cs::kOnlineThreads;
  const int64_t tile_vec = cs::online_tile_vec(threads, vpt);
  int stages = t.stages;
  const int64_t tile_bytes = tile_vec * 16;
  if (!t.stages) {
    // Rows that fit the ring stay resident (one HBM read); longer ones are
    // fetched twice. The wide shape takes the deepest ring that fits; the
    // others 8 stages (8 against 4 on the default shape: +3 to +7% at 65536
    // to 100000 columns, -1% at 131072).
    stages = vpt == 1 ? max_stages_for(tile_bytes) : kOnlineDefaultStages;
  }
  stages = std::max(1, std::min(stages, max_stages_for(tile_bytes)));
  const int smem = (int)(stages * tile_bytes) + cs::online_tail_bytes(stages);
  void* fn = vpt == 1 ? reinterpret_cast<void*>(&cs::online_kernel<1>) : reinterpret_cast<void*>(&cs::online_kernel<2>);
  int per_sm = 0;
  CS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem));
  if (per_sm < 1) return CS_ERR_UNSUPPORTED;
  const int64_t total_rows = g.batch * g.rows;
  lp->kernel = CS_KERNEL_ONLINE;
  lp->units = total_rows;
  lp->grid = (int)std::min<int64_t>(total_rows, (int64_t)d.sms * per_sm);
  lp->block = threads;
  lp->smem = smem;
  lp->stages = stages;
  lp->vec = vpt;
  lp->ctas_per_sm = per_sm;
  lp->on.g = g;
  lp->on.total_rows = total_rows;
  lp->on.stages = stages;
  return CS_OK;
}

int plan_narrow(const DeviceInfo& d, const Geometry& g, LaunchPlan* lp) {
  const int nvec = (g.cols + 7) / 8;
  if (nvec > 32) return CS_ERR_UNSUPPORTED;
  int lanes = 1;
  while (lanes < nvec) lanes <<= 1;
  const int64_t total_rows = g.batch * g.rows;
  const int64_t rows_per_block = 8 * (32 / lanes);
  lp->kernel = CS_KERNEL_WARP;
  lp->units = total_rows;
  lp->block = 256;
  lp->grid = (int)std::min<int64_t>((total_rows + rows_per_block - 1) / rows_per_block, (int64_t)d.sms * 8);
  lp->ctas_per_sm = 8;
  lp->narrow_lanes = lanes;
  lp->nr.g = g;
  lp->nr.total_rows = total_rows;
  return CS_OK;
}

int plan_baseline(const DeviceInfo& d, const Geometry& g, LaunchPlan* lp) {
  const int64_t total_rows = g.batch * g.rows;
  lp->kernel = CS_KERNEL_BASELINE;
  lp->units = total_rows;
  lp->block = 256;
  lp->grid = (int)std::min<int64_t>(total_rows, (int64_t)d.sms * 8);
  lp->ctas_per_sm = 8;
  lp->bl.g = g;
  lp->bl.total_rows = total_rows;
  return CS_OK;
}

// Resolve AUTO for a concrete geometry and build the launch plan.
int make_plan_uncached(const DeviceInfo& d, int kernel, const Geometry& g, const Tuning& t, LaunchPlan* lp) {
  if (!is_known_kernel(kernel)) return CS_ERR_BAD_KERNEL;
  switch (kernel) {
    case CS_KERNEL_BASELINE: return plan_baseline(d, g, lp);
    case CS_KERNEL_WARP:
      if (g.cols > 32) {
        std::snprintf(t_detail, sizeof t_detail, "warp specialization requires cols<=32");
        return CS_ERR_WARP_COLS;
      }
      return plan_narrow(d, g, lp);
    case CS_KERNEL_TMA: return plan_rowres(d, g, t, false, lp);
    case CS_KERNEL_PIPELINE: return plan_rowres(d, g, t, true, lp);
    case CS_KERNEL_ONLINE: return plan_online(d, g, t, lp);
    default: break;
  }
  if (g.cols <= 32) return plan_narrow(d, g, lp);
  // The bulk-store variant: measured on B200 it is 1-6% faster than per-lane
  // stores on 4096-wide rows and level from 8192 columns up.
  const int rc = plan_rowres(d, g, t, true, lp);
  if (rc != CS_ERR_UNSUPPORTED) return rc;
  return plan_online(d, g, t, lp);
}

// Planning asks the occupancy calculator about several variants and ring
// depths (tens of microseconds of host time), while a launch of a small
// matrix takes a few microseconds on the GPU. Plans therefore depend only on
// the shape, tuning and device, and are kept per host thread: a repeat
// launch of the same shape costs a lookup plus the geometry copy.
struct PlanKey {
  const DeviceInfo* dev;
  int kernel;
  Tuning t;
  int64_t batch, batch_stride;
  int32_t rows, cols, pitch, row_offset, split_row, split_shift;
  bool operator==(const PlanKey& o) const {
    return dev == o.dev && kernel == o.kernel && t.vec == o.t.vec && t.stages == o.t.stages &&
           t.hint == o.t.hint && t.zero_tma == o.t.zero_tma &&
           t.prefetch == o.t.prefetch && batch == o.batch &&
           batch_stride == o.batch_stride && rows == o.rows && cols == o.cols && pitch == o.pitch &&
           row_offset == o.row_offset && split_row == o.split_row && split_shift == o.split_shift;
  }
};
constexpr int kPlanCacheSize = 16;
thread_local PlanKey t_plan_keys[kPlanCacheSize];
thread_local LaunchPlan t_plans[kPlanCacheSize];
thread_local int t_plan_count = 0, t_plan_next = 0;

int make_plan(const DeviceInfo& d, int kernel, const Geometry& g, const Tuning& t, LaunchPlan* lp) {
  const PlanKey key{&d, kernel, t, g.batch, g.batch_stride, g.rows, g.cols, g.pitch, g.row_offset,
                    g.split_row, g.split_shift};
  for (int i = 0; i < t_plan_count; ++i) {
    if (t_plan_keys[i] == key) {
      *lp = t_plans[i];
      lp->rr.g = g;  // pointers, scale, status word, flags and timeout of this call
      if (!lp->dyn_sched) lp->rr.g.sched = nullptr;
      lp->on.g = g;
      lp->cl.g = g;
      lp->nr.g = g;
      lp->bl.g = g;
      return CS_OK;
    }
  }
  const int rc = make_plan_uncached(d, kernel, g, t, lp);
  if (rc) return rc;
  t_plan_keys[t_plan_next] = key;
  t_plans[t_plan_next] = *lp;
  t_plan_next = (t_plan_next + 1) % kPlanCacheSize;
  if (t_plan_count < kPlanCacheSize) ++t_plan_count;
  return CS_OK;
}

// Every library kernel is launched with programmatic stream serialization:
// its CTAs may start (and set up shared memory and barriers) while the
// previous kernel in the stream finishes; the kernel waits for that kernel's
// completion (pdl_wait) before touching global memory.
template <typename Params>
cudaError_t launch_pdl(void (*kernel)(Params), int grid, int block, int smem, cudaStream_t stream,
                       const Params& p) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

int launch_plan(const LaunchPlan& lp, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  switch (lp.kernel) {
    case CS_KERNEL_TMA:
    case CS_KERNEL_PIPELINE: {
      const bool ts = lp.kernel == CS_KERNEL_PIPELINE;
      switch (lp.variant) {
#define CS_ROW_LAUNCH(i, v, t, b)                                                                   \
  case i:                                                                                           \
    e = ts ? launch_pdl(&cs::rowres_kernel<v, t, b, true>, lp.grid, lp.block, lp.smem, stream, lp.rr) \
           : launch_pdl(&cs::rowres_kernel<v, t, b, false>, lp.grid, lp.block, lp.smem, stream, lp.rr); \
    break;
        CS_ROW_VARIANTS(CS_ROW_LAUNCH)
#undef CS_ROW_LAUNCH
        default: return CS_ERR_BAD_KERNEL;
      }
      break;
    }
    case CS_KERNEL_ONLINE:
      if (lp.cluster) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)lp.grid);
        cfg.blockDim = dim3((unsigned)lp.block);
        cfg.dynamicSmemBytes = (size_t)lp.smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)lp.cl.csize;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        e = cudaLaunchKernelEx(&cfg, &cs::cluster_kernel, lp.cl);
        break;
      }
      e = lp.vec == 1 ? launch_pdl(&cs::online_kernel<1>, lp.grid, lp.block, lp.smem, stream, lp.on)
                      : launch_pdl(&cs::online_kernel<2>, lp.grid, lp.block, lp.smem, stream, lp.on);
      break;
    case CS_KERNEL_WARP: {
      void (*k)(cs::NarrowParams) = nullptr;
      switch (lp.narrow_lanes) {
        case 1: k = &cs::narrow_kernel<1>; break;
        case 2: k = &cs::narrow_kernel<2>; break;
        case 4: k = &cs::narrow_kernel<4>; break;
        case 8: k = &cs::narrow_kernel<8>; break;
        case 16: k = &cs::narrow_kernel<16>; break;
        default: k = &cs::narrow_kernel<32>; break;
      }
      e = launch_pdl(k, lp.grid, lp.block, 0, stream, lp.nr);
      break;
    }
    case CS_KERNEL_BASELINE:
      e = launch_pdl(&cs::baseline_kernel, lp.grid, lp.block, 0, stream, lp.bl);
      break;
    default:
      return CS_ERR_BAD_KERNEL;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return CS_OK;
}

// online_ring_vec: 16-byte vectors the online kernel's ring holds (stages x tile).
double modelled_bytes(int kernel, const Geometry& g, int64_t online_ring_vec) {
  const double t = geometry_causal_elements(g, g.cols);
  const double w = 2.0 * (double)g.rows * (double)g.cols;
  double per = 0;
  switch (kernel) {
    case CS_KERNEL_BASELINE: per = 6.0 * t + w; break;
    case CS_KERNEL_ONLINE: {
      // Rows longer than the ring are fetched twice.
      const int64_t resident_cols = online_ring_vec * 8;
      const double t_long = g.cols > resident_cols
                                ? std::max(0.0, t - geometry_causal_elements(g, std::min<int64_t>(g.cols, resident_cols)))
                                : 0.0;
      per = 2.0 * t + 2.0 * t_long + w;
      break;
    }
    default: per = 2.0 * t + w; break;
  }
  return per * (double)g.batch;
}

// Launch through a geometry (plans, one-shot calls and sessions share this).
int launch_geometry(int dev, int kernel, const Geometry& g, const Tuning& t, cudaStream_t stream,
                    LaunchPlan* out_plan) {
  DeviceInfo* d = nullptr;
  int rc = device_info(dev, &d);
  if (rc) return rc;
  LaunchPlan lp;
  rc = make_plan(*d, kernel, g, t, &lp);
  if (rc) return rc;
  if (out_plan) *out_plan = lp;
  const bool rowres = lp.kernel == CS_KERNEL_TMA || lp.kernel == CS_KERNEL_PIPELINE;
  if (!rowres || lp.rr.m.total_units < kMaxUnitsPerLaunch) return launch_plan(lp, stream);
  // The row-resident kernel indexes units in 32 bits: split the batch.
  const int64_t per = std::max<int64_t>(1, kMaxUnitsPerLaunch / lp.rr.m.units_per_matrix);
  for (int64_t b0 = 0; b0 < g.batch; b0 += per) {
    Geometry gc = g;
    gc.in = g.in + b0 * g.batch_stride;
    gc.out = g.out + b0 * g.batch_stride;
    gc.batch = std::min<int64_t>(per, g.batch - b0);
    LaunchPlan lc;
    rc = make_plan(*d, lp.kernel, gc, t, &lc);
    if (!rc) rc = launch_plan(lc, stream);
    if (rc) return rc;
  }
  return CS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_pointers(const void* in, const void* out) {
  if (!in || !out) return CS_ERR_NULL;
  if (!aligned16(in) || !aligned16(out)) return CS_ERR_ALIGNMENT;
  if (in == out) {
    std::snprintf(t_detail, sizeof t_detail, "in-place softmax is not supported");
    return CS_ERR_ARG;
  }
  return CS_OK;
}

int status_word_for(int dev, uint32_t** out) {
  DeviceInfo* d = nullptr;
  int rc = device_info(dev, &d);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!d->oneshot_status) {
    DeviceGuard guard(dev);
    uint32_t* p = nullptr;
    CS_CUDA(cudaMalloc(&p, 256));
    CS_CUDA(cudaMemset(p, 0, 256));
    d->oneshot_status = p;
  }
  *out = d->oneshot_status;
  return CS_OK;
}

}  // namespace

// ===========================================================================
// Plans
// ===========================================================================

struct cs_plan {
  int device = 0;
  Geometry g{};
  uint32_t* d_status = nullptr;
  Tuning tuning{};
};

struct cs_session {
  int device = 0;
  cudaStream_t streams[2] = {nullptr, nullptr};
  uint32_t* d_status = nullptr;
  unsigned long long* d_counter = nullptr;
  // host-path chunk buffers
  uint16_t* d_in[2] = {nullptr, nullptr};
  uint16_t* d_out[2] = {nullptr, nullptr};
  size_t slot_bytes = 0;
  // prepare / launch / result state
  uint16_t* p_in = nullptr;
  uint16_t* p_out = nullptr;
  size_t p_bytes = 0;
  int32_t p_rows = 0, p_cols = 0, p_pitch = 0;
  bool prepared = false;
};

namespace {

// The host path moves only causal bytes across PCIe: rows are sent in blocks
// of kHostRowBlock, each with the width of its widest (last) row, in both
// directions; rows that reach the full width go in one block. The masked
// tail of each output row past its block's width is written +0.0 by host
// threads while the copies run (disjoint bytes), instead of being copied.
constexpr int32_t kHostRowBlock = 256;
constexpr unsigned kMaxZeroThreads = 8;

// Zero `bytes` at `p` (even address) without reading the lines first: on
// x86-64, 16-byte non-temporal stores for the aligned middle (measured on the
// B200 host: ordinary stores of the 4.3 GB of tails cost ~18 ms of a 120 ms
// step next to the DMA traffic, through read-for-ownership); elsewhere memset.
void zero_bytes(uint8_t* p, size_t bytes) {
#if defined(__x86_64__)
  uint8_t* end = p + bytes;
  uint8_t* a = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
  if (a >= end) {
    std::memset(p, 0, bytes);
    return;
  }
  std::memset(p, 0, (size_t)(a - p));
  const __m128i z = _mm_setzero_si128();
  for (; a + 16 <= end; a += 16) _mm_stream_si128(reinterpret_cast<__m128i*>(a), z);
  std::memset(a, 0, (size_t)(end - a));
#else
  std::memset(p, 0, bytes);
#endif
}

template <class F>
void for_each_row_block(int32_t rows, int32_t cols, int32_t row_offset, F f) {
  int64_t tri = (int64_t)cols - 1 - row_offset;  // rows with valid < cols
  tri = tri < 0 ? 0 : (tri > rows ? rows : tri);
  for (int32_t r0 = 0; r0 < tri; r0 += kHostRowBlock) {
    const int32_t r1 = (int32_t)std::min<int64_t>(r0 + kHostRowBlock, tri);
    f(r0, r1, (int32_t)std::min<int64_t>((int64_t)row_offset + r1, cols));
  }
  if (tri < rows) f((int32_t)tri, rows, cols);
}

// Chunks of the host path: whole matrices while one fits the chunk target
// (1/8 of the job, between 8 and 256 MB of device buffer), else row blocks
// of one matrix, each launched with its absolute row offset, so that copies
// and kernels overlap on the two streams even for a single large matrix.
constexpr int64_t kChunkMinBytes = int64_t(8) << 20, kChunkMaxBytes = int64_t(256) << 20;

int32_t host_chunk_rows(int64_t batch, int32_t rows, int64_t pitch, int64_t* mats_per_chunk) {
  const int64_t mat = (int64_t)rows * pitch * 2;
  const int64_t job = batch > INT64_MAX / mat ? INT64_MAX : batch * mat;
  const int64_t target = std::min(kChunkMaxBytes, std::max(kChunkMinBytes, job / 8));
  if (mat <= target) {
    *mats_per_chunk = std::max<int64_t>(1, std::min<int64_t>(batch, target / mat));
    return rows;
  }
  *mats_per_chunk = 1;
  return (int32_t)std::max<int64_t>(1, std::min<int64_t>(rows, target / (pitch * 2)));
}

// Causal row blocks of one matrix split into chunks of rc rows.
template <class F>
void for_each_copy_block(int32_t rows, int32_t cols, int32_t row_offset, int32_t rc, F f) {
  for (int32_t r0 = 0; r0 < rows; r0 += rc) {
    const int32_t n = std::min(rc, rows - r0);
    for_each_row_block(n, cols, row_offset + r0,
                       [&](int32_t a, int32_t b, int32_t w) { f(r0 + a, r0 + b, w); });
  }
}

// Bytes one direction of the host path carries for `batch` matrices.
int64_t host_copy_bytes(int64_t batch, int32_t rows, int32_t cols, int32_t row_offset) {
  int64_t mpc = 0;
  const int32_t rc = host_chunk_rows(batch, rows, padded_pitch(cols), &mpc);
  int64_t per = 0;
  for_each_copy_block(rows, cols, row_offset, rc,
                      [&](int32_t r0, int32_t r1, int32_t w) { per += (int64_t)(r1 - r0) * w * 2; });
  return per * batch;
}

// Zero the masked tails [w, cols) of every output row on host threads.
void zero_output_tails(uint16_t* h_out, int64_t batch, int32_t rows, int32_t cols, int32_t row_offset,
                       int32_t rc, std::vector<std::thread>& pool) {
  std::vector<int32_t> width(rows);
  bool any = false;
  for_each_copy_block(rows, cols, row_offset, rc, [&](int32_t r0, int32_t r1, int32_t w) {
    for (int32_t r = r0; r < r1; ++r) width[r] = w;
    any |= w < cols;
  });
  if (!any) return;
  const int64_t total_rows = batch * rows;
  // Leave cores for the thread that issues the copies.
  const unsigned hw = std::thread::hardware_concurrency();
  unsigned nt = std::max(1u, std::min(kMaxZeroThreads, hw > 2 ? hw - 2 : 1u));
  nt = (unsigned)std::min<int64_t>(nt, total_rows);
  auto zero_share = [=](unsigned t, const std::vector<int32_t>& w) {
    for (int64_t i = total_rows * t / nt; i < total_rows * (t + 1) / nt; ++i) {
      const int32_t r = (int32_t)(i % rows);
      if (w[r] < cols)
        zero_bytes(reinterpret_cast<uint8_t*>(h_out + i * cols + w[r]), (size_t)(cols - w[r]) * 2);
    }
#if defined(__x86_64__)
    _mm_sfence();  // streaming stores visible before the thread is joined
#endif
  };
  for (unsigned t = 0; t < nt; ++t) {
    try {
      pool.emplace_back([=]() { zero_share(t, width); });
    } catch (...) {
      // No thread to be had (resource limits): this share runs here instead,
      // before the copies are issued; no exception leaves the C ABI.
      zero_share(t, width);
    }
  }
}

}  // namespace

extern "C" {

int cs_abi_version(void) { return CS_ABI_VERSION; }

const char* cs_strerror(int code) {
  switch (code) {
    case CS_OK: return "ok";
    case CS_ERR_EMPTY: return "matrix dimensions must be positive";
    case CS_ERR_WRONG_LENGTH: return "score buffer length does not match matrix dimensions";
    case CS_ERR_BAD_SCALE: return "attention scale must be finite and in [0, 1e30]";
    case CS_ERR_NON_FINITE: return "score matrix contains NaN or infinity";
    case CS_ERR_WARP_COLS: return "warp specialization requires cols<=32";
    case CS_ERR_ALIGNMENT: return "base address must be nonnull and 16-byte aligned";
    case CS_ERR_PITCH: return "pitch must be >= cols, a multiple of 8 elements and fit i32";
    case CS_ERR_BAD_KERNEL: return "unknown kernel";
    case CS_ERR_DEVICE: return "no usable sm_100 (compute capability 10.x) device";
    case CS_ERR_CUDA: return "CUDA runtime error";
    case CS_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    case CS_ERR_NULL: return "null pointer argument";
    case CS_ERR_PADDING: return "nonzero padded output";
    case CS_ERR_UNSUPPORTED: return "shape not supported by the selected kernel";
    case CS_ERR_PROBE: return "probe kernel mismatch";
    case CS_ERR_ARG: return "invalid argument";
    case CS_ERR_STATUS: return "device status word holds reserved bits";
    default: return "unknown error code";
  }
}

const char* cs_last_error_detail(void) { return t_detail; }

const char* cs_kernel_name(int kernel) {
  switch (kernel) {
    case CS_KERNEL_AUTO: return "auto";
    case CS_KERNEL_BASELINE: return "baseline";
    case CS_KERNEL_WARP: return "warp";
    case CS_KERNEL_TMA: return "tma";
    case CS_KERNEL_PIPELINE: return "pipeline";
    case CS_KERNEL_ONLINE: return "online";
    default: return nullptr;
  }
}

int cs_kernel_parse(const char* name) {
  if (!name) return CS_ERR_BAD_KERNEL;
  for (int k = CS_KERNEL_AUTO; k <= CS_KERNEL_ONLINE; ++k)
    if (std::strcmp(name, cs_kernel_name(k)) == 0) return k;
  return CS_ERR_BAD_KERNEL;
}

int cs_kernel_supports(int kernel, int64_t cols) {
  if (!is_known_kernel(kernel)) return 0;
  return kernel != CS_KERNEL_WARP || cols <= 32;
}

int cs_resolve_kernel(int kernel, int64_t rows, int64_t cols) {
  if (!is_known_kernel(kernel)) return CS_ERR_BAD_KERNEL;
  if (kernel != CS_KERNEL_AUTO) return kernel;
  if (cols <= 32) return CS_KERNEL_WARP;
  // Host-side rule equal to make_plan's: the row-resident kernel takes any
  // shape whose widest unit (a row pair, else a single row) fits one of its
  // variants (the shared-memory one takes any width) and two stages of
  // shared memory.
  Geometry g{};
  g.batch = 1;
  g.rows = (int32_t)std::min<int64_t>(rows, kI32Max);
  g.cols = (int32_t)std::min<int64_t>(cols, kI32Max);
  g.pitch = (int32_t)std::min<int64_t>(padded_pitch(cols), kI32Max - 7);
  for (bool paired : {true, false}) {
    const cs::UnitMap m = cs::make_unit_map(g, paired);
    const int64_t max_nv = rowres_max_vectors(g, m);
    const int64_t stage = (max_nv * 16 + 127) / 128 * 128;
    if (rowres_shape(max_nv, m.n_pairs > 0, 0) &&
        2 * stage + cs::rowres_tail_bytes(2) <= 232448)
      return CS_KERNEL_PIPELINE;
  }
  return CS_KERNEL_ONLINE;
}

double cs_logical_bytes(int kernel, int64_t rows, int64_t cols) {
  if (!is_known_kernel(kernel) || kernel == CS_KERNEL_AUTO || rows <= 0 || cols <= 0) return -1.0;
  Geometry g{};
  g.batch = 1;
  g.rows = (int32_t)std::min<int64_t>(rows, kI32Max);
  g.cols = (int32_t)std::min<int64_t>(cols, kI32Max);
  return modelled_bytes(kernel, g, (int64_t)kOnlineDefaultStages * cs::kOnlineTileVec);
}

double cs_roofline_bytes(int64_t rows, int64_t cols, int64_t row_offset) {
  if (rows <= 0 || cols <= 0 || row_offset < 0) return 0.0;
  return 2.0 * causal_elements(rows, cols, row_offset) + 2.0 * (double)rows * (double)cols;
}

int64_t cs_padded_pitch(int64_t cols) { return padded_pitch(cols); }

int cs_validate(int64_t batch, int64_t batch_stride, int64_t rows, int64_t cols, int64_t pitch,
                int64_t row_offset, float scale) {
  return validate_args(batch, batch_stride, rows, cols, pitch, row_offset, scale);
}

int cs_check_finite_host(const uint16_t* scores, int64_t n) {
  if (n > 0 && !scores) return CS_ERR_NULL;
  for (int64_t i = 0; i < n; ++i)
    if ((scores[i] & 0x7c00u) == 0x7c00u) return CS_ERR_NON_FINITE;
  return CS_OK;
}

int cs_status_error(uint32_t status) {
  if (status == 0) return CS_OK;
  if (status & CS_STATUS_TIMEOUT) return CS_ERR_TIMEOUT;
  std::snprintf(t_detail, sizeof t_detail, "device status word 0x%08x: reserved bits set", status);
  return CS_ERR_STATUS;
}

int cs_device_sm_count(int device) {
  DeviceInfo* d = nullptr;
  const int rc = device_info(device, &d);
  return rc ? rc : d->sms;
}

int cs_plan_create(cs_plan** plan, int device, const void* d_in, void* d_out, int64_t batch,
                   int64_t batch_stride, int32_t rows, int32_t cols, int32_t pitch, int32_t row_offset) {
  if (!plan) return CS_ERR_NULL;
  *plan = nullptr;
  int rc = validate_args(batch, batch_stride, rows, cols, pitch, row_offset, 1.0f);
  if (rc) return rc;
  rc = check_pointers(d_in, d_out);
  if (rc) return rc;
  DeviceInfo* d = nullptr;
  rc = device_info(device, &d);
  if (rc) return rc;
  cs_plan* p = new (std::nothrow) cs_plan();
  if (!p) return CS_ERR_ARG;
  p->device = device;
  p->g.in = static_cast<const uint16_t*>(d_in);
  p->g.out = static_cast<uint16_t*>(d_out);
  p->g.batch = batch;
  p->g.batch_stride = batch > 1 ? batch_stride : (int64_t)rows * pitch;
  p->g.rows = rows;
  p->g.cols = cols;
  p->g.pitch = pitch;
  p->g.row_offset = row_offset;
  p->g.timeout_ns = kDefaultTimeoutNs;
  DeviceGuard guard(device);
  cudaError_t e = cudaMalloc(&p->d_status, 256);
  if (e == cudaSuccess) e = cudaMemset(p->d_status, 0, 256);
  if (e != cudaSuccess) {
    if (p->d_status) cudaFree(p->d_status);
    delete p;
    return cuda_fail(e, "plan status word");
  }
  p->g.status = p->d_status;
  // Words 1-2 of the plan's zeroed 256-byte block: the row-resident kernel's
  // dynamic schedule (a plan's launches must not overlap, so they never share
  // the counters; the kernel leaves them zero).
  p->g.sched = p->d_status + 1;
  *plan = p;
  return CS_OK;
}

int cs_plan_set_timeout(cs_plan* plan, uint64_t timeout_ns) {
  if (!plan) return CS_ERR_NULL;
  if (timeout_ns == 0) return CS_ERR_ARG;
  plan->g.timeout_ns = timeout_ns;
  return CS_OK;
}

int cs_plan_set_row_split(cs_plan* plan, int32_t split_row, int32_t split_offset) {
  if (!plan) return CS_ERR_NULL;
  if (split_row == 0) {
    plan->g.split_row = 0;
    plan->g.split_shift = 0;
    return CS_OK;
  }
  const Geometry& g = plan->g;
  // The second block starts at or after the first one's end (absolute rows
  // increase with the local row) and stays within 32-bit row indices.
  if (split_row < 0 || split_row >= g.rows || split_offset < 0 ||
      (int64_t)split_offset < (int64_t)g.row_offset + split_row ||
      (int64_t)split_offset > kI32Max - ((int64_t)g.rows - split_row)) {
    std::snprintf(t_detail, sizeof t_detail,
                  "row split %d at absolute row %d: needs 0 < split_row < rows (%d) and a second block "
                  "starting at or after row %lld",
                  (int)split_row, (int)split_offset, (int)g.rows, (long long)g.row_offset + split_row);
    return CS_ERR_ARG;
  }
  plan->g.split_row = split_row;
  plan->g.split_shift = (int32_t)((int64_t)split_offset - g.row_offset - split_row);
  return CS_OK;
}

int cs_plan_set_tuning(cs_plan* plan, int vec_per_thread, int stages, int l2_hint, int zero_fill_tma) {
  if (!plan) return CS_ERR_NULL;
  const bool variant_pick = vec_per_thread >= 16 && vec_per_thread < 16 + kNumRowVariants;
  if (vec_per_thread != 0 && vec_per_thread != 1 && vec_per_thread != 2 && vec_per_thread != 3 &&
      vec_per_thread != 4 && vec_per_thread != 8 && !variant_pick)
    return CS_ERR_ARG;
  if (stages < 0 || stages > kMaxStages || l2_hint < -1 || l2_hint > 1) return CS_ERR_ARG;
  if (zero_fill_tma < -1 || zero_fill_tma > 1) return CS_ERR_ARG;
  plan->tuning.vec = vec_per_thread;
  plan->tuning.stages = stages;
  plan->tuning.hint = l2_hint;
  plan->tuning.zero_tma = zero_fill_tma;
  return CS_OK;
}

int cs_plan_set_prefetch(cs_plan* plan, int prefetch_units) {
  if (!plan) return CS_ERR_NULL;
  if (prefetch_units < -1 || prefetch_units > 1024) return CS_ERR_ARG;
  plan->tuning.prefetch = prefetch_units;
  return CS_OK;
}

static int plan_launch_impl(cs_plan* plan, int kernel, float scale, void* stream, uint32_t flags,
                            uint64_t timeout_ns) {
  if (!plan) return CS_ERR_NULL;
  if (!std::isfinite(scale) || !(scale >= 0.0f && scale <= CS_MAX_SCALE)) return CS_ERR_BAD_SCALE;
  Geometry g = plan->g;
  g.scale = scale;
  g.flags = flags;
  if (timeout_ns) g.timeout_ns = timeout_ns;
  DeviceGuard guard(plan->device);
  if (!guard.ok()) return CS_ERR_DEVICE;
  return launch_geometry(plan->device, kernel, g, plan->tuning, static_cast<cudaStream_t>(stream), nullptr);
}

int cs_plan_launch(cs_plan* plan, int kernel, float scale, void* stream) {
  return plan_launch_impl(plan, kernel, scale, stream, 0u, 0ull);
}

int cs_plan_launch_debug(cs_plan* plan, int kernel, float scale, void* stream, uint32_t flags,
                         uint64_t timeout_ns) {
  return plan_launch_impl(plan, kernel, scale, stream, flags, timeout_ns);
}

int cs_plan_status(cs_plan* plan, uint32_t* status) {
  if (!plan) return CS_ERR_NULL;
  DeviceGuard guard(plan->device);
  CS_CUDA(cudaDeviceSynchronize());
  uint32_t s = 0;
  CS_CUDA(cudaMemcpy(&s, plan->d_status, sizeof s, cudaMemcpyDeviceToHost));
  CS_CUDA(cudaMemset(plan->d_status, 0, sizeof s));
  if (status) *status = s;
  return cs_status_error(s);
}

int cs_plan_describe(cs_plan* plan, int kernel, cs_launch_info* info) {
  if (!plan || !info) return CS_ERR_NULL;
  DeviceInfo* d = nullptr;
  DeviceGuard guard(plan->device);
  int rc = device_info(plan->device, &d);
  if (rc) return rc;
  LaunchPlan lp;
  rc = make_plan(*d, kernel, plan->g, plan->tuning, &lp);
  if (rc) return rc;
  std::memset(info, 0, sizeof *info);
  info->kernel = lp.kernel;
  info->grid = lp.grid;
  info->block = lp.block;
  info->smem_bytes = lp.smem;
  info->stages = lp.stages;
  info->vec_per_thread = lp.vec;
  info->ctas_per_sm = lp.ctas_per_sm;
  info->launches = 1;
  info->units = lp.units;
  info->algorithmic_bytes =
      (2.0 * geometry_causal_elements(plan->g, plan->g.cols) + 2.0 * (double)plan->g.rows * plan->g.cols) *
      (double)plan->g.batch;
  info->modelled_bytes =
      modelled_bytes(lp.kernel, plan->g,
                     lp.cluster ? (int64_t)plan->g.pitch  // the whole row resident in the cluster
                     : lp.kernel == CS_KERNEL_ONLINE ? (int64_t)lp.stages * cs::online_tile_vec(lp.block, lp.vec)
                                                     : (int64_t)kOnlineDefaultStages * cs::kOnlineTileVec);
  return CS_OK;
}

void cs_plan_destroy(cs_plan* plan) {
  if (!plan) return;
  {
    DeviceGuard guard(plan->device);
    if (plan->d_status) cudaFree(plan->d_status);
  }
  delete plan;
}

int cs_softmax_batched(int kernel, const void* d_in, void* d_out, int64_t batch, int64_t batch_stride,
                       int32_t rows, int32_t cols, int32_t pitch, int32_t row_offset, float scale,
                       void* stream) {
  int rc = validate_args(batch, batch_stride, rows, cols, pitch, row_offset, scale);
  if (rc) return rc;
  rc = check_pointers(d_in, d_out);
  if (rc) return rc;
  if (!is_known_kernel(kernel)) return CS_ERR_BAD_KERNEL;
  int dev = 0;
  CS_CUDA(cudaGetDevice(&dev));
  uint32_t* status = nullptr;
  rc = status_word_for(dev, &status);
  if (rc) return rc;
  Geometry g{};
  g.in = static_cast<const uint16_t*>(d_in);
  g.out = static_cast<uint16_t*>(d_out);
  g.batch = batch;
  g.batch_stride = batch > 1 ? batch_stride : (int64_t)rows * pitch;
  g.rows = rows;
  g.cols = cols;
  g.pitch = pitch;
  g.row_offset = row_offset;
  g.scale = scale;
  g.status = status;
  g.timeout_ns = kDefaultTimeoutNs;
  return launch_geometry(dev, kernel, g, Tuning{}, static_cast<cudaStream_t>(stream), nullptr);
}

int cs_softmax(int kernel, const void* d_in, void* d_out, int32_t rows, int32_t cols, int32_t pitch,
               float scale, void* stream) {
  return cs_softmax_batched(kernel, d_in, d_out, 1, 0, rows, cols, pitch, 0, scale, stream);
}

// ===========================================================================
// One-shot launch that allocates nothing
// ===========================================================================

// The status words of cs_softmax_noalloc, one per slot. They live in the
// library's device image rather than in cudaMalloc'd memory, so that entry
// point never allocates; every GPU that loads the library holds these
// CS_NOALLOC_SLOTS * 4 = 256 bytes until the process exits. On the host the
// name only stands in for the symbol: the device address comes from
// cudaGetSymbolAddress.
static __device__ __align__(256) uint32_t g_noalloc_status[CS_NOALLOC_SLOTS];

namespace {

// Device address of g_noalloc_status on `dev`, which must be the current
// device. Looked up once per device, on that device's first call.
int noalloc_status_for(int dev, uint32_t** out) {
  DeviceInfo* d = nullptr;
  int rc = device_info(dev, &d);
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!d->noalloc_status) {
    uint32_t* p = nullptr;
    CS_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_status));
    d->noalloc_status = p;
  }
  *out = d->noalloc_status;
  return CS_OK;
}

}  // namespace

int cs_softmax_noalloc(int kernel, const void* d_in, void* d_out, int64_t batch, int64_t batch_stride,
                       int32_t rows, int32_t cols, int32_t pitch, int32_t row_offset, float scale,
                       int32_t slot, uint32_t* status, void* stream) {
  int rc = validate_args(batch, batch_stride, rows, cols, pitch, row_offset, scale);
  if (rc) return rc;
  rc = check_pointers(d_in, d_out);
  if (rc) return rc;
  if (!is_known_kernel(kernel)) return CS_ERR_BAD_KERNEL;
  if (slot < 0 || slot >= CS_NOALLOC_SLOTS) {
    std::snprintf(t_detail, sizeof t_detail,
                  "status slot %d out of range: the static status array holds %d words (slots 0..%d)",
                  (int)slot, CS_NOALLOC_SLOTS, CS_NOALLOC_SLOTS - 1);
    return CS_ERR_ARG;
  }
  int dev = 0;
  CS_CUDA(cudaGetDevice(&dev));
  uint32_t* words = nullptr;
  rc = noalloc_status_for(dev, &words);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The word keeps the bits of the last call that used this slot.
  CS_CUDA(cudaMemsetAsync(words + slot, 0, sizeof(uint32_t), s));
  Geometry g{};
  g.in = static_cast<const uint16_t*>(d_in);
  g.out = static_cast<uint16_t*>(d_out);
  g.batch = batch;
  g.batch_stride = batch > 1 ? batch_stride : (int64_t)rows * pitch;
  g.rows = rows;
  g.cols = cols;
  g.pitch = pitch;
  g.row_offset = row_offset;
  g.scale = scale;
  g.status = words + slot;
  g.timeout_ns = kDefaultTimeoutNs;
  rc = launch_geometry(dev, kernel, g, Tuning{}, s, nullptr);
  if (rc || !status) return rc;
  uint32_t word = 0;
  CS_CUDA(cudaMemcpyAsync(&word, words + slot, sizeof word, cudaMemcpyDeviceToHost, s));
  CS_CUDA(cudaStreamSynchronize(s));
  *status = word;
  return cs_status_error(word);
}

int cs_noalloc_status(int32_t slot, uint32_t* status, void* stream) {
  if (!status) return CS_ERR_NULL;
  if (slot < 0 || slot >= CS_NOALLOC_SLOTS) {
    std::snprintf(t_detail, sizeof t_detail,
                  "status slot %d out of range: the static status array holds %d words (slots 0..%d)",
                  (int)slot, CS_NOALLOC_SLOTS, CS_NOALLOC_SLOTS - 1);
    return CS_ERR_ARG;
  }
  int dev = 0;
  CS_CUDA(cudaGetDevice(&dev));
  uint32_t* words = nullptr;
  const int rc = noalloc_status_for(dev, &words);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t word = 0;
  CS_CUDA(cudaMemcpyAsync(&word, words + slot, sizeof word, cudaMemcpyDeviceToHost, s));
  CS_CUDA(cudaMemsetAsync(words + slot, 0, sizeof(uint32_t), s));
  CS_CUDA(cudaStreamSynchronize(s));
  *status = word;
  return cs_status_error(word);
}

// ===========================================================================
// Sessions
// ===========================================================================

int cs_session_create(cs_session** session, int device) {
  if (!session) return CS_ERR_NULL;
  *session = nullptr;
  DeviceInfo* d = nullptr;
  int rc = device_info(device, &d);
  if (rc) return rc;
  DeviceGuard guard(device);
  cs_session* s = new (std::nothrow) cs_session();
  if (!s) return CS_ERR_ARG;
  s->device = device;
  cudaError_t e = cudaStreamCreateWithFlags(&s->streams[0], cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->streams[1], cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&s->d_status, 256);
  if (e == cudaSuccess) e = cudaMemset(s->d_status, 0, 256);
  if (e == cudaSuccess) e = cudaMalloc(&s->d_counter, sizeof(unsigned long long));
  if (e != cudaSuccess) {
    cs_session_destroy(s);
    return cuda_fail(e, "session setup");
  }
  *session = s;
  return CS_OK;
}

void* cs_session_stream(cs_session* session) { return session ? session->streams[0] : nullptr; }

int cs_session_probe(cs_session* session) {
  if (!session) return CS_ERR_NULL;
  DeviceGuard guard(session->device);
  uint32_t* d = nullptr;
  CS_CUDA(cudaMalloc(&d, 256 * sizeof(uint32_t)));
  cs::probe_kernel<<<1, 256, 0, session->streams[0]>>>(d, 256);
  uint32_t h[256];
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpyAsync(h, d, sizeof h, cudaMemcpyDeviceToHost, session->streams[0]);
  if (e == cudaSuccess) e = cudaStreamSynchronize(session->streams[0]);
  cudaFree(d);
  if (e != cudaSuccess) return cuda_fail(e, "probe");
  for (int i = 0; i < 256; ++i)
    if (h[i] != ((uint32_t)i ^ 0x5a5a5a5au)) {
      std::snprintf(t_detail, sizeof t_detail, "probe mismatch at %d", i);
      return CS_ERR_PROBE;
    }
  return CS_OK;
}

static int session_read_status(cs_session* s) {
  uint32_t st = 0;
  CS_CUDA(cudaMemcpy(&st, s->d_status, sizeof st, cudaMemcpyDeviceToHost));
  if (st) CS_CUDA(cudaMemset(s->d_status, 0, sizeof st));
  return cs_status_error(st);
}

int64_t cs_host_copy_bytes(int64_t batch, int32_t rows, int32_t cols, int32_t row_offset) {
  if (batch <= 0 || rows <= 0 || cols <= 0 || row_offset < 0) return CS_ERR_EMPTY;
  return host_copy_bytes(batch, rows, cols, row_offset);
}

static int session_softmax_host(cs_session* session, int kernel, const uint16_t* h_in, uint16_t* h_out,
                                int64_t batch, int32_t rows, int32_t cols, int32_t row_offset,
                                float scale) {
  if (!session || !h_in || !h_out) return CS_ERR_NULL;
  const int64_t pitch = padded_pitch(cols);
  int rc = validate_args(batch, (int64_t)rows * pitch, rows, cols, pitch, row_offset, scale);
  if (rc) return rc;
  if (!is_known_kernel(kernel)) return CS_ERR_BAD_KERNEL;
  DeviceGuard guard(session->device);
  const size_t mat_host = (size_t)rows * (size_t)cols * 2;
  const size_t dpitch = (size_t)pitch * 2, hpitch = (size_t)cols * 2;
  // Chunks alternate between two streams/slots.
  int64_t mpc = 0;
  const int32_t crow = host_chunk_rows(batch, rows, pitch, &mpc);
  const size_t need = (size_t)mpc * (size_t)crow * dpitch;
  if (need > session->slot_bytes) {
    for (int i = 0; i < 2; ++i) {
      if (session->d_in[i]) cudaFree(session->d_in[i]);
      if (session->d_out[i]) cudaFree(session->d_out[i]);
      session->d_in[i] = session->d_out[i] = nullptr;
    }
    session->slot_bytes = 0;
    for (int i = 0; i < 2; ++i) {
      CS_CUDA(cudaMalloc(&session->d_in[i], need));
      CS_CUDA(cudaMalloc(&session->d_out[i], need));
    }
    session->slot_bytes = need;
  }
  // Host threads zero the output's masked tails while the copies run.
  std::vector<std::thread> zeroers;
  struct JoinAll {  // joins on every exit, including an exception
    std::vector<std::thread>& v;
    ~JoinAll() {
      for (auto& t : v)
        if (t.joinable()) t.join();
    }
  } join_all{zeroers};
  zero_output_tails(h_out, batch, rows, cols, row_offset, crow, zeroers);
  auto join = [&]() {
    for (auto& t : zeroers) t.join();
    zeroers.clear();
  };
  struct Block {
    int32_t r0, r1, w;
  };
  std::vector<Block> blocks;
  // One 3-D copy per causal row block covers the block in all n matrices of
  // a chunk (depth = matrices), so the host issues a few dozen copies per
  // chunk. Host slices are whole matrices (rows x cols); device slices are
  // the chunk's nr rows at the padded pitch.
  auto copy_blocks = [&](uint8_t* dev, const uint8_t* host, int64_t n, int32_t nr,
                         cudaMemcpyKind kind, cudaStream_t st) -> cudaError_t {
    const cudaPitchedPtr dp = make_cudaPitchedPtr(dev, dpitch, dpitch, (size_t)nr);
    const cudaPitchedPtr hp = make_cudaPitchedPtr(const_cast<uint8_t*>(host), hpitch, hpitch, (size_t)rows);
    for (const Block& k : blocks) {
      cudaMemcpy3DParms m{};
      m.srcPtr = kind == cudaMemcpyHostToDevice ? hp : dp;
      m.dstPtr = kind == cudaMemcpyHostToDevice ? dp : hp;
      m.srcPos = make_cudaPos(0, (size_t)k.r0, 0);
      m.dstPos = make_cudaPos(0, (size_t)k.r0, 0);
      m.extent = make_cudaExtent((size_t)k.w * 2, (size_t)(k.r1 - k.r0), (size_t)n);
      m.kind = kind;
      const cudaError_t e = cudaMemcpy3DAsync(&m, st);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  };
  int64_t it = 0;
  for (int64_t b0 = 0; b0 < batch; b0 += mpc) {
    const int64_t n = std::min<int64_t>(mpc, batch - b0);
    for (int32_t r0 = 0; r0 < rows; r0 += crow, ++it) {
      const int32_t nr = std::min(crow, rows - r0);
      const int slot = (int)(it & 1);
      cudaStream_t st = session->streams[slot];
      const size_t hoff = (size_t)b0 * mat_host + (size_t)r0 * hpitch;
      blocks.clear();
      for_each_row_block(nr, cols, row_offset + r0,
                         [&](int32_t a, int32_t b, int32_t w) { blocks.push_back({a, b, w}); });
      cudaError_t ce = copy_blocks(reinterpret_cast<uint8_t*>(session->d_in[slot]),
                                   reinterpret_cast<const uint8_t*>(h_in) + hoff, n, nr,
                                   cudaMemcpyHostToDevice, st);
      if (ce == cudaSuccess) {
        Geometry g{};
        g.in = session->d_in[slot];
        g.out = session->d_out[slot];
        g.batch = n;
        g.batch_stride = (int64_t)nr * pitch;
        g.rows = nr;
        g.cols = cols;
        g.pitch = (int32_t)pitch;
        g.row_offset = row_offset + r0;
        g.scale = scale;
        g.status = session->d_status;
        g.timeout_ns = kDefaultTimeoutNs;
        rc = launch_geometry(session->device, kernel, g, Tuning{}, st, nullptr);
        if (!rc)
          ce = copy_blocks(reinterpret_cast<uint8_t*>(session->d_out[slot]),
                           reinterpret_cast<uint8_t*>(h_out) + hoff, n, nr, cudaMemcpyDeviceToHost, st);
      }
      if (ce != cudaSuccess) rc = cuda_fail(ce, "host path copy");
      if (rc) {
        cudaStreamSynchronize(session->streams[0]);
        cudaStreamSynchronize(session->streams[1]);
        join();
        return rc;
      }
    }
  }
  const cudaError_t e0 = cudaStreamSynchronize(session->streams[0]);
  const cudaError_t e1 = cudaStreamSynchronize(session->streams[1]);
  join();
  if (e0 != cudaSuccess) return cuda_fail(e0, "cudaStreamSynchronize");
  if (e1 != cudaSuccess) return cuda_fail(e1, "cudaStreamSynchronize");
  return session_read_status(session);
}

int cs_session_softmax_host(cs_session* session, int kernel, const uint16_t* h_in, uint16_t* h_out,
                            int64_t batch, int32_t rows, int32_t cols, int32_t row_offset,
                            float scale) {
  try {
    return session_softmax_host(session, kernel, h_in, h_out, batch, rows, cols, row_offset, scale);
  } catch (...) {
    if (session) {  // no copy may still be writing into the caller's buffers
      cudaStreamSynchronize(session->streams[0]);
      cudaStreamSynchronize(session->streams[1]);
    }
    std::snprintf(t_detail, sizeof t_detail, "host path: out of host memory or threads");
    return CS_ERR_ARG;
  }
}

int cs_session_prepare(cs_session* session, const uint16_t* h_in, int32_t rows, int32_t cols) {
  if (!session || !h_in) return CS_ERR_NULL;
  const int64_t pitch = padded_pitch(cols);
  int rc = validate_args(1, 0, rows, cols, pitch, 0, 1.0f);
  if (rc) return rc;
  DeviceGuard guard(session->device);
  const size_t bytes = (size_t)rows * (size_t)pitch * 2;
  if (bytes > session->p_bytes) {
    if (session->p_in) cudaFree(session->p_in);
    if (session->p_out) cudaFree(session->p_out);
    session->p_in = session->p_out = nullptr;
    session->p_bytes = 0;
    CS_CUDA(cudaMalloc(&session->p_in, bytes));
    CS_CUDA(cudaMalloc(&session->p_out, bytes));
    session->p_bytes = bytes;
  }
  cudaStream_t st = session->streams[0];
  // gpu/src/driver.rs:75-79: zero padding on the input, sentinel 0xfb00 on the output.
  CS_CUDA(cudaMemsetAsync(session->p_in, 0, bytes, st));
  CS_CUDA(cudaMemcpy2DAsync(session->p_in, (size_t)pitch * 2, h_in, (size_t)cols * 2, (size_t)cols * 2,
                            (size_t)rows, cudaMemcpyHostToDevice, st));
  const int64_t n = (int64_t)rows * pitch;
  cs::fill_u16_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, st>>>(session->p_out, n, 0xfb00u);
  CS_CUDA(cudaGetLastError());
  CS_CUDA(cudaStreamSynchronize(st));
  session->p_rows = rows;
  session->p_cols = cols;
  session->p_pitch = (int32_t)pitch;
  session->prepared = true;
  return CS_OK;
}

int cs_session_launch(cs_session* session, int kernel, float scale) {
  if (!session) return CS_ERR_NULL;
  if (!session->prepared) return CS_ERR_ARG;
  if (!std::isfinite(scale) || !(scale >= 0.0f && scale <= CS_MAX_SCALE)) return CS_ERR_BAD_SCALE;
  DeviceGuard guard(session->device);
  Geometry g{};
  g.in = session->p_in;
  g.out = session->p_out;
  g.batch = 1;
  g.batch_stride = (int64_t)session->p_rows * session->p_pitch;
  g.rows = session->p_rows;
  g.cols = session->p_cols;
  g.pitch = session->p_pitch;
  g.scale = scale;
  g.status = session->d_status;
  g.timeout_ns = kDefaultTimeoutNs;
  return launch_geometry(session->device, kernel, g, Tuning{}, session->streams[0], nullptr);
}

int cs_session_result(cs_session* session, uint16_t* h_out) {
  if (!session || !h_out) return CS_ERR_NULL;
  if (!session->prepared) return CS_ERR_ARG;
  DeviceGuard guard(session->device);
  cudaStream_t st = session->streams[0];
  CS_CUDA(cudaStreamSynchronize(st));
  int rc = session_read_status(session);
  if (rc) return rc;
  const int32_t rows = session->p_rows, cols = session->p_cols, pitch = session->p_pitch;
  if (pitch > cols) {
    CS_CUDA(cudaMemsetAsync(session->d_counter, 0, sizeof(unsigned long long), st));
    const int64_t n = (int64_t)rows * (pitch - cols);
    cs::padding_check_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, st>>>(
        session->p_out, rows, cols, pitch, session->d_counter);
    CS_CUDA(cudaGetLastError());
    unsigned long long bad = 0;
    CS_CUDA(cudaMemcpyAsync(&bad, session->d_counter, sizeof bad, cudaMemcpyDeviceToHost, st));
    CS_CUDA(cudaStreamSynchronize(st));
    if (bad) {
      std::snprintf(t_detail, sizeof t_detail, "%llu nonzero padded outputs", bad);
      return CS_ERR_PADDING;
    }
  }
  CS_CUDA(cudaMemcpy2DAsync(h_out, (size_t)cols * 2, session->p_out, (size_t)pitch * 2, (size_t)cols * 2,
                            (size_t)rows, cudaMemcpyDeviceToHost, st));
  CS_CUDA(cudaStreamSynchronize(st));
  return CS_OK;
}

void cs_session_destroy(cs_session* session) {
  if (!session) return;
  {
    DeviceGuard guard(session->device);
    for (int i = 0; i < 2; ++i) {
      if (session->streams[i]) cudaStreamSynchronize(session->streams[i]);
    }
    for (int i = 0; i < 2; ++i) {
      if (session->d_in[i]) cudaFree(session->d_in[i]);
      if (session->d_out[i]) cudaFree(session->d_out[i]);
      if (session->streams[i]) cudaStreamDestroy(session->streams[i]);
    }
    if (session->p_in) cudaFree(session->p_in);
    if (session->p_out) cudaFree(session->p_out);
    if (session->d_status) cudaFree(session->d_status);
    if (session->d_counter) cudaFree(session->d_counter);
  }
  delete session;
}

int cs_host_register(void* ptr, size_t bytes) {
  if (!ptr) return CS_ERR_NULL;
  CS_CUDA(cudaHostRegister(ptr, bytes, cudaHostRegisterDefault));
  return CS_OK;
}

int cs_host_unregister(void* ptr) {
  if (!ptr) return CS_ERR_NULL;
  CS_CUDA(cudaHostUnregister(ptr));
  return CS_OK;
}

}  // extern "C"
