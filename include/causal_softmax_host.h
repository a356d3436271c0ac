/*
 * causal_softmax_host.h — GPU-independent host surface of the B200 fused
 * causal softmax (input patterns, seeded workload generator, numerical
 * verifier, output self-check, bench statistics and the CLI configuration).
 *
 * It is the C++ counterpart of the reference project's host crate
 * (host/src/lib.rs in R-P-Padhi/GB200-SM100A-TMA-Fused-Causal-Attention-Softmax;
 * citations below are paths inside that project), exported through the same
 * shared library as causal_softmax.h. Nothing here touches a GPU.
 */
#ifndef CAUSAL_SOFTMAX_HOST_H
#define CAUSAL_SOFTMAX_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* host/src/lib.rs:185-216 (enum Pattern). */
typedef enum cs_pattern {
    CS_PATTERN_ZEROS = 0,
    CS_PATTERN_RAMP = 1,
    CS_PATTERN_ALTERNATING = 2,
    CS_PATTERN_SPIKES = 3,
    CS_PATTERN_EXTREME = 4,
    CS_PATTERN_TINY = 5,
    CS_PATTERN_RANDOM = 6
} cs_pattern;

/* host/src/lib.rs:205-215 (Pattern::name); NULL for an unknown value. */
const char *cs_pattern_name(int pattern);

/* IEEE binary32 -> binary16, round to nearest even, subnormals, overflow to
 * infinity (reference/src/lib.rs:48-83), and binary16 -> binary32 exactly
 * (reference/src/lib.rs:30-45). */
uint16_t cs_f32_to_half(float x);
float cs_half_to_f32(uint16_t h);

/* host/src/lib.rs:218-256 (make_input): rows*cols dense halves of `pattern`,
 * xorshift32 state seeded with `seed` (advanced once per element). */
int cs_make_input(uint16_t *out, int64_t rows, int64_t cols, int pattern, uint32_t seed);

/* Seeded synthetic workloads of the five benchmark configurations. Element
 * (b, r, c) is a pure function of (seed, first_batch + b, first_row + r, c), from a
 * counter-based splitmix64 generator (Vigna's published mixer), so any
 * sub-block can be regenerated independently:
 *   1: half(N(0,1) * 4)                         (4096 x 4096 single matrix)
 *   2: half(U(-8, 8))                           (odd / narrow shapes)
 *   3: half(N(0,1) * 8); 1% of entries +-60000; in every row r >= 1 the
 *      row's causal maximum is copied to two distinct columns c <= r (ties)
 *   4: half(N(0,1) * 3)                         (batched multi-head)
 *   5: half(N(0,1) * 2 + 0.001 * c)             (long context)
 * Normal draws use Box-Muller on two 24-bit uniforms. The output has the
 * strided layout (batch_stride, pitch); padding columns are written 0.
 * first_batch / first_row are the absolute matrix and row of local matrix 0,
 * row 0, so a head shard or a row-block shard regenerates exactly its part of
 * the full workload (ties included). `threads` <= 0 uses all hardware threads. */
int cs_generate(uint16_t *out, int config, uint64_t seed, int64_t batch, int64_t batch_stride,
                int64_t rows, int64_t cols, int64_t pitch, int64_t first_batch, int64_t first_row,
                int threads);

/* host/src/lib.rs:258-328 (Accuracy, VerifyError, verify) for dense
 * rows x cols outputs; returns one of CS_VERIFY_*. */
enum {
    CS_VERIFY_OK = 0,
    CS_VERIFY_LENGTH = 1,
    CS_VERIFY_NON_FINITE = 2,
    CS_VERIFY_NEGATIVE = 3,
    CS_VERIFY_MASK = 4,
    CS_VERIFY_ELEMENT = 5,
    CS_VERIFY_ROW_SUM = 6
};
typedef struct cs_accuracy {
    float max_abs;
    float max_relative;
    float max_row_sum_error;
    int64_t index; /* failing element (or row for ROW_SUM), -1 if none */
    float got;
    float want;
} cs_accuracy;
int cs_verify(const uint16_t *got, size_t got_len, const uint16_t *expected, size_t expected_len,
              size_t rows, size_t cols, cs_accuracy *acc);

/* Oracle-free self-check of a strided output (what the CLI can check with
 * no reference output): masked columns and padding are 0x0000, valid entries
 * are finite and non-negative, and |row sum - 1| <= rowsum_tol (f64 sum). */
typedef struct cs_self_check {
    int64_t rows_checked;
    int64_t mask_violations;
    int64_t nonfinite_or_negative;
    int64_t rowsum_violations;
    double max_rowsum_err;
} cs_self_check;
int cs_check_output(const uint16_t *out, int64_t batch, int64_t batch_stride, int64_t rows,
                    int64_t cols, int64_t pitch, int64_t row_offset, double rowsum_tol,
                    cs_self_check *report);

/* host/src/lib.rs:330-407 (BenchStats): nearest-rank tails, population SD. */
typedef struct cs_bench_stats {
    int64_t samples;
    double min_ms, median_ms, p95_ms, p99_ms, max_ms, mean_ms, stddev_ms, cv_pct;
} cs_bench_stats;
int cs_bench_stats_from_ms(const double *ms, int64_t n, cs_bench_stats *out);

/* host/src/lib.rs:383-406 (BenchStats::report): one "kernel=... GBps..."
 * line into buf (NUL-terminated, truncated to buflen). Returns the length
 * the full line needs. */
int cs_bench_report(const cs_bench_stats *s, const char *name, int64_t rows, int64_t cols,
                    double logical_bytes, char *buf, size_t buflen);

/* host/src/lib.rs:67-183 (Action, Config): flags --probe --gpu-tests
 * --gpu-stress --bench --bench-suite --no-verify --stress --rows --cols
 * --scale --kernel --iterations --warmup, plus --config N (1..5) --batch B
 * --seed S --gpus G --pitch P. */
typedef enum cs_action {
    CS_ACTION_RUN = 0,
    CS_ACTION_PROBE = 1,
    CS_ACTION_GPU_TESTS = 2,
    CS_ACTION_GPU_STRESS = 3,
    CS_ACTION_BENCH = 4,
    CS_ACTION_BENCH_SUITE = 5,
    CS_ACTION_HELP = 6
} cs_action;
typedef struct cs_config {
    int32_t action;
    int32_t kernel;
    int64_t rows, cols, pitch, batch;
    float scale;
    int32_t iterations, warmup;
    int32_t verify;
    int32_t config;   /* 0: reference Random pattern input; 1..5 generator configs */
    uint64_t seed;
    int32_t gpus;
} cs_config;
/* Parses argv[0..argc) (no program name). Returns 0, or -1 with a message in err. */
int cs_config_parse(int argc, const char *const *argv, cs_config *out, char *err, size_t errlen);
/* host/src/lib.rs:143-168 on an already filled config; 0 or -1 with message. */
int cs_config_validate(const cs_config *c, char *err, size_t errlen);
/* host/src/lib.rs:178-182 (Config::help). */
const char *cs_config_help(void);

#ifdef __cplusplus
}
#endif

#endif /* CAUSAL_SOFTMAX_HOST_H */
