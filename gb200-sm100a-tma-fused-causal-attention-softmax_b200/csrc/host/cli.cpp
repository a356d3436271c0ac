// csm — command-line driver over the C ABI, mirroring the reference CLI
// (gpu/src/driver.rs:386-428 main_entry; flags host/src/lib.rs:103-142).
//
//   csm [--rows M --cols N --scale F --kernel K]      run + self-check
//   csm --probe                                        probe kernel
//   csm --gpu-tests | --gpu-stress                     shape x pattern x kernel matrix
//   csm --bench [--iterations N --warmup N]            CUDA-event timing, BENCH line
//   csm --bench-suite                                  shapes, queue depth, transfers, device
//                                                      copy, patterns x scales, streams
//
// Checks here are oracle-free (masked entries 0x0000, finite non-negative
// values, row sums within 2e-3 of 1); comparison against the CPU oracle lives
// in the test suite.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "causal_softmax.h"
#include "causal_softmax_host.h"

namespace {

int fail(const char* what, int rc) {
  std::fprintf(stderr, "%s: %s (%s)\n", what, cs_strerror(rc), cs_last_error_detail());
  return 1;
}

struct DeviceMatrix {
  uint16_t* in = nullptr;
  uint16_t* out = nullptr;
  int64_t rows = 0, cols = 0, pitch = 0, batch = 1;
  ~DeviceMatrix() {
    if (in) cudaFree(in);
    if (out) cudaFree(out);
  }
};

// Host input (pattern or generator config), padded to the pitch.
std::vector<uint16_t> make_host(const cs_config& c, int64_t pitch) {
  std::vector<uint16_t> h((size_t)(c.batch * c.rows * pitch), 0);
  if (c.config >= 1) {
    cs_generate(h.data(), c.config, c.seed, c.batch, c.rows * pitch, c.rows, c.cols, pitch, 0, 0, 0);
  } else {
    std::vector<uint16_t> dense((size_t)(c.rows * c.cols));
    for (int64_t b = 0; b < c.batch; ++b) {
      cs_make_input(dense.data(), c.rows, c.cols, CS_PATTERN_RANDOM, (uint32_t)c.seed);
      for (int64_t r = 0; r < c.rows; ++r)
        std::memcpy(&h[(size_t)((b * c.rows + r) * pitch)], &dense[(size_t)(r * c.cols)],
                    (size_t)c.cols * 2);
    }
  }
  return h;
}

int upload(const cs_config& c, DeviceMatrix& m) {
  m.rows = c.rows;
  m.cols = c.cols;
  m.batch = c.batch;
  m.pitch = c.pitch ? c.pitch : cs_padded_pitch(c.cols);
  const size_t bytes = (size_t)(m.batch * m.rows * m.pitch) * 2;
  if (cudaMalloc(&m.in, bytes) != cudaSuccess || cudaMalloc(&m.out, bytes) != cudaSuccess)
    return fail("cudaMalloc", CS_ERR_CUDA);
  const std::vector<uint16_t> h = make_host(c, m.pitch);
  if (cudaMemcpy(m.in, h.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail("upload", CS_ERR_CUDA);
  return 0;
}

int self_check(const DeviceMatrix& m, const char* name, double* max_err) {
  std::vector<uint16_t> h((size_t)(m.batch * m.rows * m.pitch));
  if (cudaMemcpy(h.data(), m.out, h.size() * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail("download", CS_ERR_CUDA);
  cs_self_check r{};
  const int bad = cs_check_output(h.data(), m.batch, m.rows * m.pitch, m.rows, m.cols, m.pitch, 0,
                                  2e-3, &r);
  if (max_err) *max_err = r.max_rowsum_err;
  if (bad) {
    std::printf("FAIL %s %lldx%lld: mask=%lld nonfinite/negative=%lld rowsum=%lld (max err %.3g)\n",
                name, (long long)m.rows, (long long)m.cols, (long long)r.mask_violations,
                (long long)r.nonfinite_or_negative, (long long)r.rowsum_violations, r.max_rowsum_err);
    return 1;
  }
  return 0;
}

int run_once(const cs_config& c, int kernel, DeviceMatrix& m) {
  cs_plan* plan = nullptr;
  int rc = cs_plan_create(&plan, 0, m.in, m.out, m.batch, m.rows * m.pitch, (int32_t)m.rows,
                          (int32_t)m.cols, (int32_t)m.pitch, 0);
  if (rc) return fail("cs_plan_create", rc);
  rc = cs_plan_launch(plan, kernel, c.scale, nullptr);
  uint32_t st = 0;
  if (!rc) rc = cs_plan_status(plan, &st);
  cs_plan_destroy(plan);
  return rc ? fail("launch", rc) : 0;
}

int action_run(const cs_config& c) {
  DeviceMatrix m;
  if (upload(c, m)) return 1;
  const int kernel = cs_resolve_kernel(c.kernel, c.rows, c.cols);
  if (run_once(c, kernel, m)) return 1;
  if (!c.verify) {
    std::printf("launched %s %lldx%lld (checks disabled)\n", cs_kernel_name(kernel),
                (long long)c.rows, (long long)c.cols);
    return 0;
  }
  double err = 0;
  if (self_check(m, cs_kernel_name(kernel), &err)) return 1;
  std::printf("PASS %s %lldx%lld scale=%g max_row_sum_err=%.6f\n", cs_kernel_name(kernel),
              (long long)c.rows, (long long)c.cols, c.scale, err);
  return 0;
}

// gpu/src/driver.rs:250-331 shape lists, patterns and scales, oracle-free.
int action_gpu_tests(const cs_config& base, bool stress) {
  static const int quick[][2] = {{1, 1}, {1, 8}, {2, 17}, {3, 31}, {4, 32}, {5, 33}, {7, 64},
                                 {8, 127}, {9, 256}, {10, 257}, {13, 513}, {17, 1024}, {33, 9}, {64, 65}};
  static const int more[][2] = {{1, 129}, {2, 255}, {3, 256}, {4, 257}, {5, 511}, {6, 512},
                                {7, 513}, {8, 1025}, {15, 2048}, {16, 16}, {31, 31}, {32, 32},
                                {33, 33}, {64, 128}, {65, 256}, {127, 512}, {129, 8192}, {257, 257}};
  const int n_shapes = stress ? 18 : 14;
  const int patterns_stress[] = {0, 1, 2, 3, 4, 5, 6}, patterns_quick[] = {0, 3, 6};
  const float scales_stress[] = {0.0f, 0.125f, 0.5f, 1.0f, 1.0e30f}, scales_quick[] = {0.125f};
  int passed = 0;
  for (int si = 0; si < n_shapes; ++si) {
    const int rows = stress ? more[si][0] : quick[si][0];
    const int cols = stress ? more[si][1] : quick[si][1];
    for (int pi = 0; pi < (stress ? 7 : 3); ++pi) {
      const int pattern = stress ? patterns_stress[pi] : patterns_quick[pi];
      for (int kernel = CS_KERNEL_BASELINE; kernel <= CS_KERNEL_ONLINE; ++kernel) {
        if (!cs_kernel_supports(kernel, cols)) continue;
        for (int sc = 0; sc < (stress ? 5 : 1); ++sc) {
          cs_config c = base;
          c.rows = rows;
          c.cols = cols;
          c.pitch = 0;
          c.batch = 1;
          c.config = 0;
          c.scale = stress ? scales_stress[sc] : scales_quick[sc];
          DeviceMatrix m;
          m.rows = rows;
          m.cols = cols;
          m.pitch = cs_padded_pitch(cols);
          const size_t bytes = (size_t)(rows * m.pitch) * 2;
          if (cudaMalloc(&m.in, bytes) != cudaSuccess || cudaMalloc(&m.out, bytes) != cudaSuccess)
            return fail("cudaMalloc", CS_ERR_CUDA);
          std::vector<uint16_t> dense((size_t)rows * cols), padded(bytes / 2, 0);
          cs_make_input(dense.data(), rows, cols, pattern, 0x13579bdf);
          for (int r = 0; r < rows; ++r)
            std::memcpy(&padded[(size_t)r * m.pitch], &dense[(size_t)r * cols], (size_t)cols * 2);
          cudaMemcpy(m.in, padded.data(), bytes, cudaMemcpyHostToDevice);
          if (run_once(c, kernel, m) || self_check(m, cs_kernel_name(kernel), nullptr)) {
            std::printf("FAIL %s %dx%d %s scale=%g\n", cs_kernel_name(kernel), rows, cols,
                        cs_pattern_name(pattern), c.scale);
            return 1;
          }
          ++passed;
        }
      }
    }
  }
  std::printf("PASS GPU self-checks: %d cases\n", passed);
  return 0;
}

int bench_kernel(const cs_config& c, int kernel, DeviceMatrix& m) {
  cs_plan* plan = nullptr;
  int rc = cs_plan_create(&plan, 0, m.in, m.out, m.batch, m.rows * m.pitch, (int32_t)m.rows,
                          (int32_t)m.cols, (int32_t)m.pitch, 0);
  if (rc) return fail("cs_plan_create", rc);
  cudaStream_t st;
  cudaStreamCreate(&st);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  for (int i = 0; i < c.warmup && !rc; ++i) rc = cs_plan_launch(plan, kernel, c.scale, st);
  std::vector<double> ms;
  for (int i = 0; i < c.iterations && !rc; ++i) {
    cudaEventRecord(a, st);
    rc = cs_plan_launch(plan, kernel, c.scale, st);
    cudaEventRecord(b, st);
    cudaEventSynchronize(b);
    float t = 0;
    cudaEventElapsedTime(&t, a, b);
    ms.push_back(t);
  }
  uint32_t status = 0;
  if (!rc) rc = cs_plan_status(plan, &status);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaStreamDestroy(st);
  cs_plan_destroy(plan);
  if (rc) return fail("bench launch", rc);
  cs_bench_stats s{};
  cs_bench_stats_from_ms(ms.data(), (int64_t)ms.size(), &s);
  char line[512];
  const double bytes = cs_roofline_bytes(m.rows, m.cols, 0) * (double)m.batch;
  cs_bench_report(&s, cs_kernel_name(kernel), m.rows, m.cols, bytes, line, sizeof line);
  std::printf("BENCH %s batch=%lld roofline_bytes=%.0f\n", line, (long long)m.batch, bytes);
  return 0;
}

int action_bench(const cs_config& c) {
  DeviceMatrix m;
  if (upload(c, m)) return 1;
  for (int kernel = CS_KERNEL_BASELINE; kernel <= CS_KERNEL_ONLINE; ++kernel) {
    if (c.kernel != CS_KERNEL_AUTO && kernel != c.kernel) continue;
    if (!cs_kernel_supports(kernel, c.cols)) continue;
    if (c.verify && (run_once(c, kernel, m) || self_check(m, cs_kernel_name(kernel), nullptr)))
      return 1;
    if (bench_kernel(c, kernel, m)) return 1;
  }
  std::printf("Timing: CUDA events around each launch (single launches; launch latency included)\n");
  return 0;
}

// ---------------------------------------------------------------- bench suite
// The categories of gpu/src/driver/bench.rs:139-369 over the C ABI: shapes,
// launch queue depth, host transfers, device copy, patterns x scales, and
// concurrent streams. Kernel timings are CUDA events; transfers and
// concurrency are host wall clock. Self-checks are oracle-free.

int upload_pattern(int rows, int cols, int pattern, uint32_t seed, DeviceMatrix& m) {
  m.rows = rows;
  m.cols = cols;
  m.batch = 1;
  m.pitch = cs_padded_pitch(cols);
  const size_t bytes = (size_t)(rows * m.pitch) * 2;
  if (cudaMalloc(&m.in, bytes) != cudaSuccess || cudaMalloc(&m.out, bytes) != cudaSuccess)
    return fail("cudaMalloc", CS_ERR_CUDA);
  std::vector<uint16_t> dense((size_t)rows * cols), padded(bytes / 2, 0);
  cs_make_input(dense.data(), rows, cols, pattern, seed);
  for (int r = 0; r < rows; ++r)
    std::memcpy(&padded[(size_t)r * m.pitch], &dense[(size_t)r * cols], (size_t)cols * 2);
  if (cudaMemcpy(m.in, padded.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail("upload", CS_ERR_CUDA);
  return 0;
}

// Event time per launch over `queued` back-to-back launches, `samples` times.
int event_stats(cs_plan* plan, int kernel, float scale, cudaStream_t st, int warmup, int samples,
                int queued, cs_bench_stats* out) {
  int rc = 0;
  for (int i = 0; i < warmup && !rc; ++i) rc = cs_plan_launch(plan, kernel, scale, st);
  if (rc) return fail("warm-up launch", rc);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  std::vector<double> ms;
  for (int i = 0; i < samples && !rc; ++i) {
    cudaEventRecord(a, st);
    for (int q = 0; q < queued && !rc; ++q) rc = cs_plan_launch(plan, kernel, scale, st);
    cudaEventRecord(b, st);
    cudaEventSynchronize(b);
    float t = 0;
    cudaEventElapsedTime(&t, a, b);
    ms.push_back((double)t / queued);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  uint32_t status = 0;
  if (!rc) rc = cs_plan_status(plan, &status);
  if (rc) return fail("timed launch", rc);
  return cs_bench_stats_from_ms(ms.data(), (int64_t)ms.size(), out) ? fail("stats", CS_ERR_ARG) : 0;
}

int make_plan_for(const DeviceMatrix& m, cs_plan** plan) {
  const int rc = cs_plan_create(plan, 0, m.in, m.out, 1, m.rows * m.pitch, (int32_t)m.rows,
                                (int32_t)m.cols, (int32_t)m.pitch, 0);
  return rc ? fail("cs_plan_create", rc) : 0;
}

void print_bench(const char* prefix, const cs_bench_stats& s, const char* name, int64_t rows,
                 int64_t cols, double bytes, const char* suffix) {
  char line[512];
  cs_bench_report(&s, name, rows, cols, bytes, line, sizeof line);
  std::printf("BENCH %s %s%s\n", prefix, line, suffix ? suffix : "");
}

double host_ms_since(const std::chrono::steady_clock::time_point& t0) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

int suite_shapes(const cs_config& c) {
  std::vector<std::pair<int, int>> cases = {{1, 1},      {31, 31},     {32, 32},    {64, 64},
                                            {128, 257},  {256, 256},   {512, 512},  {1024, 1024},
                                            {128, 4096}, {4096, 128},  {2048, 2048}, {4096, 4096}};
  cases.push_back({(int)c.rows, (int)c.cols});
  if (c.rows >= 8192 || c.cols >= 8192) cases.push_back({8192, 8192});
  std::sort(cases.begin(), cases.end());
  cases.erase(std::unique(cases.begin(), cases.end()), cases.end());
  cudaStream_t st;
  cudaStreamCreate(&st);
  for (const auto& rc : cases) {
    DeviceMatrix m;
    if (upload_pattern(rc.first, rc.second, CS_PATTERN_RANDOM, 0x73817cdeu, m)) return 1;
    double base_ms = 0;
    for (int kernel = CS_KERNEL_BASELINE; kernel <= CS_KERNEL_ONLINE; ++kernel) {
      if (c.kernel != CS_KERNEL_AUTO && kernel != c.kernel) continue;
      if (!cs_kernel_supports(kernel, m.cols)) continue;
      cs_config one = c;
      if (c.verify && (run_once(one, kernel, m) || self_check(m, cs_kernel_name(kernel), nullptr))) return 1;
      cs_plan* plan = nullptr;
      if (make_plan_for(m, &plan)) return 1;
      cs_bench_stats s{};
      const int bad = event_stats(plan, kernel, c.scale, st, c.warmup, c.iterations, 1, &s);
      cs_plan_destroy(plan);
      if (bad) return 1;
      if (kernel == CS_KERNEL_BASELINE) base_ms = s.median_ms;
      char rel[64] = "";
      if (base_ms > 0 && s.median_ms > 0) std::snprintf(rel, sizeof rel, " speedup_vs_baseline=%.3f", base_ms / s.median_ms);
      print_bench("category=shape clock=cuda_event", s, cs_kernel_name(kernel), m.rows, m.cols,
                  cs_logical_bytes(kernel, m.rows, m.cols), rel);
    }
  }
  cudaStreamDestroy(st);
  return 0;
}

int suite_queue(const cs_config& c) {
  const int rows = (int)std::min<int64_t>(c.rows, 1024), cols = (int)std::min<int64_t>(c.cols, 1024);
  cudaStream_t st;
  cudaStreamCreate(&st);
  for (int kernel = CS_KERNEL_BASELINE; kernel <= CS_KERNEL_ONLINE; ++kernel) {
    if (c.kernel != CS_KERNEL_AUTO && kernel != c.kernel) continue;
    if (!cs_kernel_supports(kernel, cols)) continue;
    DeviceMatrix m;
    if (upload_pattern(rows, cols, CS_PATTERN_RANDOM, 0x513e79a2u, m)) return 1;
    cs_plan* plan = nullptr;
    if (make_plan_for(m, &plan)) return 1;
    for (int queued : {1, 4, 16, 64}) {
      cs_bench_stats s{};
      if (event_stats(plan, kernel, c.scale, st, c.warmup, c.iterations, queued, &s)) {
        cs_plan_destroy(plan);
        return 1;
      }
      char prefix[96];
      std::snprintf(prefix, sizeof prefix, "category=queue clock=cuda_event queued=%d", queued);
      print_bench(prefix, s, cs_kernel_name(kernel), rows, cols, cs_logical_bytes(kernel, rows, cols), nullptr);
    }
    cs_plan_destroy(plan);
  }
  cudaStreamDestroy(st);
  return 0;
}

int suite_transfers(const cs_config& c) {
  const int kernel = cs_resolve_kernel(c.kernel, c.rows, c.cols);
  DeviceMatrix m;
  if (upload_pattern((int)c.rows, (int)c.cols, CS_PATTERN_RANDOM, 0x11ba4ff2u, m)) return 1;
  const size_t bytes = (size_t)(m.rows * m.pitch) * 2;
  uint16_t *h_in = nullptr, *h_out = nullptr;
  if (cudaMallocHost(&h_in, bytes) != cudaSuccess || cudaMallocHost(&h_out, bytes) != cudaSuccess)
    return fail("cudaMallocHost", CS_ERR_CUDA);
  cudaMemcpy(h_in, m.in, bytes, cudaMemcpyDeviceToHost);
  cs_plan* plan = nullptr;
  if (make_plan_for(m, &plan)) return 1;
  cudaStream_t st;
  cudaStreamCreate(&st);
  std::vector<double> h2d, d2h, full;
  int rc = 0;
  for (int i = 0; i < c.warmup + c.iterations && !rc; ++i) {
    auto t = std::chrono::steady_clock::now();
    cudaMemcpyAsync(m.in, h_in, bytes, cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    const double a = host_ms_since(t);
    t = std::chrono::steady_clock::now();
    cudaMemcpyAsync(h_out, m.out, bytes, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    const double b = host_ms_since(t);
    t = std::chrono::steady_clock::now();
    cudaMemcpyAsync(m.in, h_in, bytes, cudaMemcpyHostToDevice, st);
    rc = cs_plan_launch(plan, kernel, c.scale, st);
    cudaMemcpyAsync(h_out, m.out, bytes, cudaMemcpyDeviceToHost, st);
    cudaStreamSynchronize(st);
    const double f = host_ms_since(t);
    if (i >= c.warmup) {
      h2d.push_back(a);
      d2h.push_back(b);
      full.push_back(f);
    }
  }
  uint32_t status = 0;
  if (!rc) rc = cs_plan_status(plan, &status);
  cs_plan_destroy(plan);
  cudaStreamDestroy(st);
  cudaFreeHost(h_in);
  cudaFreeHost(h_out);
  if (rc) return fail("transfer launch", rc);
  if (c.verify && self_check(m, cs_kernel_name(kernel), nullptr)) return 1;
  const double pb = (double)bytes;
  const struct {
    const char* stage;
    const std::vector<double>* t;
    double traffic;
  } stages[] = {{"h2d", &h2d, pb}, {"d2h", &d2h, pb},
                {"h2d_kernel_d2h", &full, 2.0 * pb + cs_logical_bytes(kernel, m.rows, m.cols)}};
  for (const auto& x : stages) {
    cs_bench_stats s{};
    cs_bench_stats_from_ms(x.t->data(), (int64_t)x.t->size(), &s);
    char prefix[96];
    std::snprintf(prefix, sizeof prefix, "category=transfer stage=%s clock=host_wall", x.stage);
    print_bench(prefix, s, cs_kernel_name(kernel), m.rows, m.cols, x.traffic, nullptr);
  }
  return 0;
}

int suite_device_copy(const cs_config& c) {
  DeviceMatrix m;
  if (upload_pattern((int)c.rows, (int)c.cols, CS_PATTERN_RANDOM, 0xbb6bf14du, m)) return 1;
  const size_t bytes = (size_t)(m.rows * m.pitch) * 2;
  cudaStream_t st;
  cudaStreamCreate(&st);
  for (int i = 0; i < c.warmup; ++i) cudaMemcpyAsync(m.out, m.in, bytes, cudaMemcpyDeviceToDevice, st);
  cudaStreamSynchronize(st);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  std::vector<double> ms;
  for (int i = 0; i < c.iterations; ++i) {
    cudaEventRecord(a, st);
    cudaMemcpyAsync(m.out, m.in, bytes, cudaMemcpyDeviceToDevice, st);
    cudaEventRecord(b, st);
    cudaEventSynchronize(b);
    float t = 0;
    cudaEventElapsedTime(&t, a, b);
    ms.push_back(t);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaStreamDestroy(st);
  if (cudaGetLastError() != cudaSuccess) return fail("device copy", CS_ERR_CUDA);
  cs_bench_stats s{};
  cs_bench_stats_from_ms(ms.data(), (int64_t)ms.size(), &s);
  // One copy reads one pitched matrix and writes another.
  print_bench("category=device_copy clock=cuda_event", s, "d2d_memcpy", m.rows, m.cols, 2.0 * (double)bytes, nullptr);
  return 0;
}

int suite_patterns(const cs_config& c) {
  const int rows = (int)std::min<int64_t>(c.rows, 256), cols = (int)std::min<int64_t>(c.cols, 256);
  cudaStream_t st;
  cudaStreamCreate(&st);
  for (int pattern : {CS_PATTERN_ZEROS, CS_PATTERN_RAMP, CS_PATTERN_ALTERNATING, CS_PATTERN_SPIKES,
                      CS_PATTERN_EXTREME, CS_PATTERN_RANDOM}) {
    DeviceMatrix m;
    if (upload_pattern(rows, cols, pattern, 0xd3ad87c1u, m)) return 1;
    for (float scale : {0.0f, 0.125f, 1.0f, 1.0e30f}) {
      for (int kernel = CS_KERNEL_BASELINE; kernel <= CS_KERNEL_ONLINE; ++kernel) {
        if (c.kernel != CS_KERNEL_AUTO && kernel != c.kernel) continue;
        if (!cs_kernel_supports(kernel, cols)) continue;
        cs_config one = c;
        one.scale = scale;
        if (c.verify && (run_once(one, kernel, m) || self_check(m, cs_kernel_name(kernel), nullptr))) return 1;
        cs_plan* plan = nullptr;
        if (make_plan_for(m, &plan)) return 1;
        cs_bench_stats s{};
        const int bad = event_stats(plan, kernel, scale, st, std::min(c.warmup, 3), std::min(c.iterations, 12),
                                    1, &s);
        cs_plan_destroy(plan);
        if (bad) return 1;
        char prefix[128];
        std::snprintf(prefix, sizeof prefix, "category=pattern pattern=%s scale=%g clock=cuda_event",
                      cs_pattern_name(pattern), scale);
        print_bench(prefix, s, cs_kernel_name(kernel), rows, cols, cs_logical_bytes(kernel, rows, cols), nullptr);
      }
    }
  }
  cudaStreamDestroy(st);
  return 0;
}

int suite_concurrency(const cs_config& c) {
  const int kernel = cs_resolve_kernel(c.kernel, c.rows, c.cols);
  const int rows = (int)std::min<int64_t>(c.rows, 512);
  const int cols = (int)std::min<int64_t>(c.cols, kernel == CS_KERNEL_WARP ? 32 : 512);
  const int queued = 4;
  double base = 0;
  for (int count : {1, 2, 4, 8}) {
    // Fresh non-blocking streams and distinct buffers: no output sharing.
    std::vector<DeviceMatrix> ms(count);
    std::vector<cs_plan*> plans(count, nullptr);
    std::vector<cudaStream_t> sts(count);
    int rc = 0;
    for (int i = 0; i < count && !rc; ++i) {
      cudaStreamCreateWithFlags(&sts[i], cudaStreamNonBlocking);
      rc = upload_pattern(rows, cols, CS_PATTERN_RANDOM, 0x58ee7719u, ms[i]) || make_plan_for(ms[i], &plans[i]);
    }
    for (int w = 0; w < c.warmup && !rc; ++w)
      for (int i = 0; i < count && !rc; ++i) rc = cs_plan_launch(plans[i], kernel, c.scale, sts[i]);
    for (int i = 0; i < count; ++i) cudaStreamSynchronize(sts[i]);
    std::vector<double> wall;
    for (int it = 0; it < c.iterations && !rc; ++it) {
      const auto t = std::chrono::steady_clock::now();
      for (int i = 0; i < count && !rc; ++i)
        for (int q = 0; q < queued && !rc; ++q) rc = cs_plan_launch(plans[i], kernel, c.scale, sts[i]);
      for (int i = 0; i < count; ++i) cudaStreamSynchronize(sts[i]);
      wall.push_back(host_ms_since(t));
    }
    for (int i = 0; i < count && !rc; ++i) {
      uint32_t status = 0;
      rc = cs_plan_status(plans[i], &status);
      if (!rc && c.verify) rc = self_check(ms[i], cs_kernel_name(kernel), nullptr) ? CS_ERR_ARG : 0;
    }
    for (int i = 0; i < count; ++i) {
      cs_plan_destroy(plans[i]);
      cudaStreamDestroy(sts[i]);
    }
    if (rc) return fail("concurrency", rc);
    cs_bench_stats s{};
    cs_bench_stats_from_ms(wall.data(), (int64_t)wall.size(), &s);
    const double calls_per_s = count * queued / (s.median_ms / 1e3);
    if (base == 0) base = calls_per_s;
    std::printf("BENCH category=concurrency clock=host_wall streams=%d calls_per_stream=%d kernel=%s "
                "rows=%d cols=%d n=%lld batch_p50_ms=%.5f batch_p95_ms=%.5f batch_p99_ms=%.5f "
                "kernels_per_s=%.2f throughput_speedup=%.3f approx_logical_GBps=%.2f\n",
                count, queued, cs_kernel_name(kernel), rows, cols, (long long)s.samples, s.median_ms,
                s.p95_ms, s.p99_ms, calls_per_s, calls_per_s / base,
                calls_per_s * cs_logical_bytes(kernel, rows, cols) / 1e9);
  }
  return 0;
}

int action_bench_suite(const cs_config& c) {
  int dev = 0;
  cudaDeviceProp prop{};
  cudaGetDevice(&dev);
  cudaGetDeviceProperties(&prop, dev);
  std::printf("BENCH hardware=%s sms=%d clock=CUDA_event_and_host_wall verify=%d warmup=%lld "
              "repetitions=%lld\n", prop.name, prop.multiProcessorCount, (int)c.verify,
              (long long)c.warmup, (long long)c.iterations);
  if (suite_shapes(c) || suite_queue(c) || suite_transfers(c) || suite_device_copy(c) ||
      suite_patterns(c) || suite_concurrency(c))
    return 1;
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  cs_config c{};
  char err[1024];
  if (cs_config_parse(argc - 1, argv + 1, &c, err, sizeof err) != 0) {
    const bool help = c.action == CS_ACTION_HELP;
    std::fprintf(help ? stdout : stderr, "%s\n", err);
    return help ? 0 : 2;
  }
  if (c.gpus != 1) std::fprintf(stderr, "note: csm drives one GPU; use bench.py under torchrun for more\n");
  switch (c.action) {
    case CS_ACTION_PROBE: {
      cs_session* s = nullptr;
      int rc = cs_session_create(&s, 0);
      if (!rc) rc = cs_session_probe(s);
      cs_session_destroy(s);
      if (rc) return fail("probe", rc);
      std::printf("PASS probe: all 256 lanes\n");
      return 0;
    }
    case CS_ACTION_GPU_TESTS: return action_gpu_tests(c, false);
    case CS_ACTION_GPU_STRESS: return action_gpu_tests(c, true);
    case CS_ACTION_BENCH: return action_bench(c);
    case CS_ACTION_BENCH_SUITE: return action_bench_suite(c);
    default: return action_run(c);
  }
}
