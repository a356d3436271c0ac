// GPU-independent host surface: patterns, workload generator, verifier,
// output self-check, bench statistics and CLI configuration.
// C++ counterpart of host/src/lib.rs; declarations in causal_softmax_host.h.
//
// Built with -ffp-contract=off so binary32 expressions round exactly as the
// reference's Rust code does (no fused multiply-add contraction).
#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "causal_softmax.h"
#include "causal_softmax_host.h"

namespace {

uint32_t f32_bits(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  return b;
}

float bits_f32(uint32_t b) {
  float x;
  std::memcpy(&x, &b, 4);
  return x;
}

// Vigna's splitmix64 finaliser (public-domain published algorithm).
inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

inline uint64_t row_key(uint64_t seed, int64_t b, int64_t abs_row) {
  return splitmix64(splitmix64(seed + 0x632BE59BD9B4E019ull * (uint64_t)b) + (uint64_t)abs_row);
}

// Box-Muller on two 24-bit uniforms from one 64-bit hash; u1 in (0, 1].
inline double normal_from(uint64_t h) {
  const double u1 = (double)((h >> 40) + 1) * (1.0 / 16777216.0);
  const double u2 = (double)((h >> 16) & 0xFFFFFFu) * (1.0 / 16777216.0);
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

inline double uniform01(uint64_t h) { return (double)(h >> 11) * (1.0 / 9007199254740992.0); }

int resolve_threads(int threads) {
  if (threads > 0) return std::min(threads, 1024);
  const unsigned hw = std::thread::hardware_concurrency();
  return hw ? (int)std::min(hw, 256u) : 1;
}

template <typename F>
void parallel_rows(int64_t n, int threads, F&& fn) {
  threads = (int)std::min<int64_t>(std::max(threads, 1), std::max<int64_t>(n, 1));
  if (threads <= 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve((size_t)threads);
  const int64_t per = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int64_t a = t * per, e = std::min(n, a + per);
    if (a >= e) break;
    try {
      pool.emplace_back([&fn, a, e] { fn(a, e); });
    } catch (...) {
      fn(a, e);  // no thread to be had: this range runs on the caller's thread
    }
  }
  for (auto& th : pool) th.join();
}

void set_err(char* err, size_t len, const std::string& msg) {
  if (!err || !len) return;
  std::snprintf(err, len, "%s", msg.c_str());
}

// Strict unsigned parse (Rust usize::from_str: optional '+', digits only).
bool parse_u64(const char* s, uint64_t* out) {
  if (!s || !*s) return false;
  if (*s == '+') ++s;
  if (!*s) return false;
  uint64_t v = 0;
  for (; *s; ++s) {
    if (*s < '0' || *s > '9') return false;
    const uint64_t d = (uint64_t)(*s - '0');
    if (v > (UINT64_MAX - d) / 10) return false;
    v = v * 10 + d;
  }
  *out = v;
  return true;
}

bool parse_f32(const char* s, float* out) {
  if (!s || !*s) return false;
  errno = 0;
  char* end = nullptr;
  const float v = std::strtof(s, &end);
  if (end == s || *end != '\0') return false;
  *out = v;  // out-of-range values become +-inf, rejected by validation
  return true;
}

}  // namespace

extern "C" {

const char* cs_pattern_name(int pattern) {
  switch (pattern) {
    case CS_PATTERN_ZEROS: return "zeros";
    case CS_PATTERN_RAMP: return "ramp";
    case CS_PATTERN_ALTERNATING: return "alternating";
    case CS_PATTERN_SPIKES: return "spikes";
    case CS_PATTERN_EXTREME: return "extreme";
    case CS_PATTERN_TINY: return "tiny";
    case CS_PATTERN_RANDOM: return "random";
    default: return nullptr;
  }
}

float cs_half_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t exp = ((uint32_t)h >> 10) & 31u;
  const uint32_t frac = (uint32_t)h & 1023u;
  uint32_t bits;
  if (exp == 0 && frac == 0) {
    bits = sign;
  } else if (exp == 0) {
    const uint32_t shift = (uint32_t)__builtin_clz(frac) - 21u;
    bits = sign | ((113u - shift) << 23) | (((frac << shift) & 1023u) << 13);
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (frac << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (frac << 13);
  }
  return bits_f32(bits);
}

uint16_t cs_f32_to_half(float x) {
  const uint32_t bits = f32_bits(x);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  const int32_t exp = (int32_t)((bits >> 23) & 255u);
  const uint32_t mant = bits & 0x7fffffu;
  if (exp == 255) return (uint16_t)(sign | (mant ? 0x7e00u : 0x7c00u));
  if (exp == 0) return sign;
  const int32_t e = exp - 112;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return sign;
    const uint32_t v = mant | 0x800000u, shift = (uint32_t)(14 - e);
    const uint32_t rem = v & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    uint32_t r = v >> shift;
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
  }
  uint32_t m = mant >> 13;
  const uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) ++m;
  return (uint16_t)(sign | (uint16_t)(((uint32_t)e << 10) + m));
}

int cs_make_input(uint16_t* out, int64_t rows, int64_t cols, int pattern, uint32_t seed) {
  if (!out) return CS_ERR_NULL;
  if (rows <= 0 || cols <= 0) return CS_ERR_EMPTY;
  if (!cs_pattern_name(pattern)) return CS_ERR_ARG;
  uint32_t state = seed;
  const int64_t n = rows * cols;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t r = i / cols, c = i % cols;
    state ^= state << 13;
    state ^= state >> 17;
    state ^= state << 5;
    float v = 0.0f;
    switch (pattern) {
      case CS_PATTERN_ZEROS: v = 0.0f; break;
      case CS_PATTERN_RAMP: v = ((float)c - (float)r) * 0.125f; break;
      case CS_PATTERN_ALTERNATING: v = (c % 2 == 0) ? -11.0f : 11.0f; break;
      case CS_PATTERN_SPIKES: v = (c == std::min(r, cols - 1)) ? 28.0f : -23.0f; break;
      case CS_PATTERN_EXTREME: v = (c % 5 == 0) ? 65000.0f : -65000.0f; break;
      case CS_PATTERN_TINY: v = (float)(c % 11) * 0.00005f - 0.00025f; break;
      default: v = ((float)(state >> 16) / 65536.0f - 0.5f) * 32.0f; break;
    }
    out[i] = cs_f32_to_half(v);
  }
  return CS_OK;
}

int cs_generate(uint16_t* out, int config, uint64_t seed, int64_t batch, int64_t batch_stride,
                int64_t rows, int64_t cols, int64_t pitch, int64_t first_batch, int64_t first_row,
                int threads) {
  if (!out) return CS_ERR_NULL;
  if (config < 1 || config > 5) return CS_ERR_ARG;
  if (batch <= 0 || rows <= 0 || cols <= 0) return CS_ERR_EMPTY;
  if (pitch < cols) return CS_ERR_PITCH;
  if (first_row < 0 || first_batch < 0) return CS_ERR_ARG;
  if (batch > 1 && batch_stride < rows * pitch) return CS_ERR_WRONG_LENGTH;
  const int64_t stride = batch > 1 ? batch_stride : rows * pitch;
  parallel_rows(batch * rows, resolve_threads(threads), [&](int64_t a, int64_t e) {
    for (int64_t t = a; t < e; ++t) {
      const int64_t b = t / rows, r = t % rows, abs_row = first_row + r;
      uint16_t* y = out + b * stride + r * pitch;
      const uint64_t rk = row_key(seed, first_batch + b, abs_row);
      for (int64_t c = 0; c < cols; ++c) {
        const uint64_t h = splitmix64(rk + (uint64_t)c);
        double v;
        switch (config) {
          case 1: v = normal_from(h) * 4.0; break;
          case 2: v = -8.0 + 16.0 * uniform01(h); break;
          case 3: {
            const uint64_t h2 = splitmix64(h ^ 0xD1B54A32D192ED03ull);
            if (h2 % 100 == 0)
              v = ((h2 >> 32) & 1u) ? 60000.0 : -60000.0;
            else
              v = normal_from(h) * 8.0;
            break;
          }
          case 4: v = normal_from(h) * 3.0; break;
          default: v = normal_from(h) * 2.0 + 0.001 * (double)c; break;
        }
        y[c] = cs_f32_to_half((float)v);
      }
      for (int64_t c = cols; c < pitch; ++c) y[c] = 0;
      if (config == 3 && abs_row >= 1) {
        const int64_t valid = std::min(abs_row + 1, cols);
        if (valid >= 2) {
          int64_t arg = 0;
          float best = cs_half_to_f32(y[0]);
          for (int64_t c = 1; c < valid; ++c) {
            const float f = cs_half_to_f32(y[c]);
            if (f > best) { best = f; arg = c; }
          }
          const uint16_t mbits = y[arg];
          const uint64_t hk = splitmix64(rk ^ 0x8CB92BA72F3D8DD7ull);
          const int64_t c1 = (int64_t)(hk % (uint64_t)valid);
          const int64_t c2 = (c1 + 1 + (int64_t)((hk >> 32) % (uint64_t)(valid - 1))) % valid;
          y[c1] = mbits;
          y[c2] = mbits;
        }
      }
    }
  });
  return CS_OK;
}

int cs_verify(const uint16_t* got, size_t got_len, const uint16_t* expected, size_t expected_len,
              size_t rows, size_t cols, cs_accuracy* acc) {
  cs_accuracy m{0.0f, 0.0f, 0.0f, -1, 0.0f, 0.0f};
  size_t n = 0;
  if (got_len != expected_len || __builtin_mul_overflow(rows, cols, &n) || n != got_len) {
    if (acc) *acc = m;
    return CS_VERIFY_LENGTH;
  }
  if (n && (!got || !expected)) return CS_VERIFY_LENGTH;
  int code = CS_VERIFY_OK;
  for (size_t row = 0; row < rows && code == CS_VERIFY_OK; ++row) {
    float sum = 0.0f;
    for (size_t col = 0; col < cols; ++col) {
      const size_t i = row * cols + col;
      const float g = cs_half_to_f32(got[i]), w = cs_half_to_f32(expected[i]);
      if (!std::isfinite(g)) { code = CS_VERIFY_NON_FINITE; m.index = (int64_t)i; break; }
      if (g < 0.0f) { code = CS_VERIFY_NEGATIVE; m.index = (int64_t)i; break; }
      if (col > row && got[i] != 0) { code = CS_VERIFY_MASK; m.index = (int64_t)i; break; }
      const float err = std::fabs(g - w);
      m.max_abs = std::max(m.max_abs, err);
      if (w > 0.0001f) m.max_relative = std::max(m.max_relative, err / w);
      if (err > 0.003f + 0.003f * std::fabs(w)) {
        code = CS_VERIFY_ELEMENT;
        m.index = (int64_t)i;
        m.got = g;
        m.want = w;
        break;
      }
      sum += g;
    }
    if (code != CS_VERIFY_OK) break;
    const float rs = std::fabs(sum - 1.0f);
    m.max_row_sum_error = std::max(m.max_row_sum_error, rs);
    if (rs > 0.02f) {
      code = CS_VERIFY_ROW_SUM;
      m.index = (int64_t)row;
      m.got = sum;
    }
  }
  if (acc) *acc = m;
  return code;
}

int cs_check_output(const uint16_t* out, int64_t batch, int64_t batch_stride, int64_t rows,
                    int64_t cols, int64_t pitch, int64_t row_offset, double rowsum_tol,
                    cs_self_check* report) {
  if (!out || !report) return CS_ERR_NULL;
  if (batch <= 0 || rows <= 0 || cols <= 0) return CS_ERR_EMPTY;
  if (pitch < cols) return CS_ERR_PITCH;
  const int64_t stride = batch > 1 ? batch_stride : rows * pitch;
  cs_self_check r{0, 0, 0, 0, 0.0};
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < rows; ++i) {
      const uint16_t* y = out + b * stride + i * pitch;
      const int64_t valid = std::min(row_offset + i + 1, cols);
      double sum = 0.0;
      for (int64_t c = 0; c < pitch; ++c) {
        if (c >= valid) {
          if (y[c] != 0) ++r.mask_violations;
          continue;
        }
        const float f = cs_half_to_f32(y[c]);
        if (!std::isfinite(f) || (y[c] & 0x8000u)) ++r.nonfinite_or_negative;
        else sum += (double)f;
      }
      const double e = std::fabs(sum - 1.0);
      r.max_rowsum_err = std::max(r.max_rowsum_err, e);
      if (!(e <= rowsum_tol)) ++r.rowsum_violations;
      ++r.rows_checked;
    }
  *report = r;
  return (r.mask_violations || r.nonfinite_or_negative || r.rowsum_violations) ? 1 : 0;
}

int cs_bench_stats_from_ms(const double* ms, int64_t n, cs_bench_stats* out) {
  if (!out) return CS_ERR_NULL;
  if (n <= 0 || !ms) return CS_ERR_EMPTY;
  std::vector<double> v(ms, ms + n);
  for (double x : v)
    if (!std::isfinite(x) || x < 0.0) return CS_ERR_ARG;
  std::sort(v.begin(), v.end());
  double mean = 0.0;
  for (double x : v) mean += x;
  mean /= (double)n;
  double var = 0.0;
  for (double x : v) var += (x - mean) * (x - mean);
  var /= (double)n;
  const double sd = std::sqrt(var);
  out->samples = n;
  out->min_ms = v[0];
  out->median_ms = (n % 2 == 0) ? (v[n / 2 - 1] + v[n / 2]) / 2.0 : v[n / 2];
  out->p95_ms = v[(n * 95 + 99) / 100 - 1];
  out->p99_ms = v[(n * 99 + 99) / 100 - 1];
  out->max_ms = v[n - 1];
  out->mean_ms = mean;
  out->stddev_ms = sd;
  out->cv_pct = mean > 0.0 ? 100.0 * sd / mean : 0.0;
  return CS_OK;
}

int cs_bench_report(const cs_bench_stats* s, const char* name, int64_t rows, int64_t cols,
                    double logical_bytes, char* buf, size_t buflen) {
  if (!s || !name) return CS_ERR_NULL;
  const double sec = s->median_ms / 1000.0;
  const double gbps = s->median_ms > 0.0 ? logical_bytes / sec / 1e9 : 0.0;
  const double melems = s->median_ms > 0.0 ? (double)rows * (double)cols / sec / 1e6 : 0.0;
  return std::snprintf(buf, buf ? buflen : 0,
                       "kernel=%s rows=%lld cols=%lld n=%lld min_ms=%.5f median_ms=%.5f p95_ms=%.5f "
                       "p99_ms=%.5f max_ms=%.5f mean_ms=%.5f stddev_ms=%.5f cv_pct=%.2f "
                       "approx_logical_GBps=%.2f Melem_per_s=%.2f",
                       name, (long long)rows, (long long)cols, (long long)s->samples, s->min_ms,
                       s->median_ms, s->p95_ms, s->p99_ms, s->max_ms, s->mean_ms, s->stddev_ms,
                       s->cv_pct, gbps, melems);
}

const char* cs_config_help(void) {
  return "--probe | --gpu-tests | --gpu-stress | --bench | --bench-suite [--rows M] [--cols N] "
         "[--scale F] [--kernel auto|baseline|warp|tma|pipeline|online] [--iterations N] "
         "[--warmup N] [--stress] [--no-verify] [--config 1..5] [--batch B] [--pitch P] "
         "[--seed S] [--gpus 1|2|4|8]";
}

int cs_config_validate(const cs_config* c, char* err, size_t errlen) {
  if (!c) return -1;
  if (c->rows == 0 || c->cols == 0 || c->rows < 0 || c->cols < 0) {
    set_err(err, errlen, "rows and cols must be positive");
    return -1;
  }
  const int64_t i32 = 2147483647;
  if (c->rows > i32 || c->cols > i32) {
    set_err(err, errlen, "dimensions exceed i32 TMA coordinates");
    return -1;
  }
  const int64_t padded = (c->cols + 7) & ~int64_t(7);
  if (padded > i32) {
    set_err(err, errlen, "padded pitch exceeds device i32 indexing");
    return -1;
  }
  int64_t tmp;
  if (__builtin_mul_overflow(c->rows, c->cols, &tmp) || __builtin_mul_overflow(c->rows, padded, &tmp)) {
    set_err(err, errlen, "matrix size overflow");
    return -1;
  }
  if (!std::isfinite(c->scale) || !(c->scale >= 0.0f && c->scale <= CS_MAX_SCALE)) {
    set_err(err, errlen, "scale must be finite and in [0, 1e30]");
    return -1;
  }
  if (c->iterations <= 0 || c->iterations > 100000 || c->warmup < 0 || c->warmup > 10000) {
    set_err(err, errlen, "invalid benchmark repetition count");
    return -1;
  }
  if (!cs_kernel_supports(c->kernel, c->cols)) {
    set_err(err, errlen, "warp specialization requires cols <= 32");
    return -1;
  }
  if (c->pitch != 0 && (c->pitch < c->cols || (c->pitch & 7) != 0 || c->pitch > i32)) {
    set_err(err, errlen, "pitch must be >= cols and a multiple of 8");
    return -1;
  }
  if (c->batch < 1 || c->config < 0 || c->config > 5) {
    set_err(err, errlen, "invalid batch or config");
    return -1;
  }
  if (c->gpus != 1 && c->gpus != 2 && c->gpus != 4 && c->gpus != 8) {
    set_err(err, errlen, "gpus must be 1, 2, 4 or 8");
    return -1;
  }
  return 0;
}

int cs_config_parse(int argc, const char* const* argv, cs_config* out, char* err, size_t errlen) {
  if (!out) return -1;
  cs_config c{};
  c.action = CS_ACTION_RUN;
  c.kernel = CS_KERNEL_AUTO;
  c.rows = 4096;
  c.cols = 4096;
  c.pitch = 0;
  c.batch = 1;
  c.scale = 0.125f;
  c.iterations = 20;
  c.warmup = 5;
  c.verify = 1;
  c.config = 0;
  c.seed = 0x13579bdfull;
  c.gpus = 1;
  for (int i = 0; i < argc; ++i) {
    const std::string key = argv[i] ? argv[i] : "";
    if (key == "--probe") c.action = CS_ACTION_PROBE;
    else if (key == "--gpu-tests") c.action = CS_ACTION_GPU_TESTS;
    else if (key == "--gpu-stress") c.action = CS_ACTION_GPU_STRESS;
    else if (key == "--bench") c.action = CS_ACTION_BENCH;
    else if (key == "--bench-suite") c.action = CS_ACTION_BENCH_SUITE;
    else if (key == "--no-verify") c.verify = 0;
    else if (key == "--stress") c.rows = c.cols = 8192;
    else if (key == "--help" || key == "-h") {
      set_err(err, errlen, cs_config_help());
      out->action = CS_ACTION_HELP;
      return -1;
    } else if (key == "--rows" || key == "--cols" || key == "--scale" || key == "--kernel" ||
               key == "--iterations" || key == "--warmup" || key == "--config" || key == "--batch" ||
               key == "--seed" || key == "--gpus" || key == "--pitch") {
      if (i + 1 >= argc || !argv[i + 1]) {
        set_err(err, errlen, "missing value for " + key);
        return -1;
      }
      const char* v = argv[++i];
      uint64_t u = 0;
      float f = 0.0f;
      const std::string name = key.substr(2);
      if (key == "--scale") {
        if (!parse_f32(v, &f)) { set_err(err, errlen, "invalid scale"); return -1; }
        c.scale = f;
      } else if (key == "--kernel") {
        const int k = cs_kernel_parse(v);
        if (k < 0) { set_err(err, errlen, std::string("unknown kernel: ") + v); return -1; }
        c.kernel = k;
      } else {
        if (!parse_u64(v, &u)) { set_err(err, errlen, "invalid " + name); return -1; }
        if (key == "--seed") { c.seed = u; continue; }
        if (u > (uint64_t)INT64_MAX) { set_err(err, errlen, "invalid " + name); return -1; }
        const int64_t s = (int64_t)u;
        if (key == "--rows") c.rows = s;
        else if (key == "--cols") c.cols = s;
        else if (key == "--pitch") c.pitch = s;
        else if (key == "--batch") c.batch = s;
        else if (s > 2147483647) { set_err(err, errlen, "invalid " + name); return -1; }
        else if (key == "--iterations") c.iterations = (int32_t)s;
        else if (key == "--warmup") c.warmup = (int32_t)s;
        else if (key == "--config") c.config = (int32_t)s;
        else c.gpus = (int32_t)s;
      }
    } else {
      set_err(err, errlen, "unknown flag: " + key + "\n" + cs_config_help());
      return -1;
    }
  }
  if (cs_config_validate(&c, err, errlen) != 0) return -1;
  *out = c;
  return 0;
}

}  // extern "C"
