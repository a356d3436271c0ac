// csm — command-line driver over the C ABI, mirroring the reference CLI
// (gpu/src/driver.rs:386-428 main_entry; flags host/src/lib.rs:103-142).
//
//   csm [--rows M --cols N --scale F --kernel K]      run + self-check
//   csm --probe                                        probe kernel
//   csm --gpu-tests | --gpu-stress                     shape x pattern x kernel matrix
//   csm --bench [--iterations N --warmup N]            CUDA-event timing, BENCH line
//   csm --bench-suite                                  shape sweep, one BENCH line each
//
// Checks here are oracle-free (masked entries 0x0000, finite non-negative
// values, row sums within 2e-3 of 1); comparison against the CPU oracle lives
// in the test suite.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
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

int action_bench_suite(const cs_config& base) {
  static const int shapes[][2] = {{4096, 32}, {1000, 1037}, {2048, 2048}, {4096, 4096},
                                  {8192, 8192}, {128, 65536}};
  for (const auto& s : shapes) {
    cs_config c = base;
    c.rows = s[0];
    c.cols = s[1];
    c.pitch = 0;
    c.batch = 1;
    c.kernel = CS_KERNEL_AUTO;
    DeviceMatrix m;
    if (upload(c, m)) return 1;
    for (int kernel = CS_KERNEL_BASELINE; kernel <= CS_KERNEL_ONLINE; ++kernel)
      if (cs_kernel_supports(kernel, c.cols) && bench_kernel(c, kernel, m)) return 1;
  }
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
