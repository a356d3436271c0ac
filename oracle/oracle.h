/*
 * CPU oracle for the fused causal softmax — TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference project's CPU specification
 * (reference/src/lib.rs), its online-kernel arithmetic model
 * (reference/src/online.rs) and its numerical verifier (host/src/lib.rs:280-328),
 * plus an FP64 oracle rounded to half for the stricter acceptance check.
 *
 * Only the test suite, the smoke check and the CPU-baseline leg of the bench
 * may load this library. The product path (the CUDA library) never links it.
 *
 * Parity pin: every known-answer test in reference/src/lib.rs:154-362,
 * reference/src/online.rs:63-123 and host/src/lib.rs:502-529 is re-run against
 * this restatement by tests/test_oracle.py (values transcribed with file:line
 * citations in tests/golden/reference_known_answers.json). The reference is
 * Rust and cannot be built in this image, so it is the pin, not a side-by-side run.
 */
#ifndef CS_ORACLE_H
#define CS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ShapeError codes, reference/src/lib.rs:8-27. */
enum {
    OR_OK = 0,
    OR_EMPTY = 1,
    OR_WRONG_LENGTH = 2,
    OR_BAD_SCALE = 3,
    OR_NON_FINITE = 4,
};

/* VerifyError codes, host/src/lib.rs:264-272. */
enum {
    OR_VERIFY_OK = 0,
    OR_VERIFY_LENGTH = 1,
    OR_VERIFY_NON_FINITE = 2,
    OR_VERIFY_NEGATIVE = 3,
    OR_VERIFY_MASK = 4,
    OR_VERIFY_ELEMENT = 5,
    OR_VERIFY_ROW_SUM = 6,
};

#define OR_MAX_SCALE 1.0e30f /* reference/src/lib.rs:5 */

float or_half_to_f32(uint16_t h);     /* reference/src/lib.rs:30-45 */
uint16_t or_f32_to_half(float x);     /* reference/src/lib.rs:48-83 */
uint16_t or_f64_to_half(double x);    /* RNE double -> half, for the FP64 oracle */

/* reference/src/lib.rs:110-129. `len` is the buffer length in elements;
 * rows*cols overflow reports OR_WRONG_LENGTH like checked_mul does. */
int or_validate(const uint16_t *scores, size_t len, size_t rows, size_t cols, float scale);

/* reference/src/lib.rs:85-108: dense rows x cols, f32 math with expf. */
int or_causal_softmax(const uint16_t *scores, size_t len, size_t rows, size_t cols,
                      float scale, uint16_t *out);

/* reference/src/online.rs:5-17 (exported for the butterfly known-answer test). */
void or_butterfly(const float in[32], int maximum, float out[32]);

/* reference/src/online.rs:19-61: the online-kernel arithmetic model. */
int or_tiled_online_softmax(const uint16_t *scores, size_t len, size_t rows, size_t cols,
                            float scale, uint16_t *out);

/* reference/src/lib.rs:132-152. */
size_t or_padded_pitch(size_t cols);
void or_pad(const uint16_t *scores, size_t rows, size_t cols, uint16_t *out);
void or_unpad(const uint16_t *padded, size_t rows, size_t cols, uint16_t *out);

/*
 * Strided generalisation of reference/src/lib.rs:85-108 used to check the GPU
 * library's batched / pitched / row-block-shard launches:
 *   matrix b, local row i has absolute causal row (row_offset + i);
 *   valid = min(row_offset + i + 1, cols); columns [valid, pitch) are written 0.
 * Arithmetic per row is exactly the reference's (f32, expf, sequential sum).
 * `threads` > 1 splits rows over POSIX threads (results are identical).
 * Input validation (finite values, scale range) is the caller's job here.
 */
int or_causal_softmax_strided(const uint16_t *in, uint16_t *out, int64_t batch,
                              int64_t batch_stride, int64_t rows, int64_t cols,
                              int64_t pitch, int64_t row_offset, float scale, int threads);

/* Same layout, FP64 arithmetic (reference/src/lib.rs:279-300), RNE to half. */
int or_causal_softmax_f64_strided(const uint16_t *in, uint16_t *out, int64_t batch,
                                  int64_t batch_stride, int64_t rows, int64_t cols,
                                  int64_t pitch, int64_t row_offset, float scale, int threads);

/* host/src/lib.rs:259-328 verifier (dense rows x cols). */
typedef struct {
    float max_abs;
    float max_relative;
    float max_row_sum_error;
    int64_t index; /* element or row index of the failure, -1 if none */
    float got;
    float want;
} or_accuracy;

int or_verify(const uint16_t *got, const uint16_t *expected, size_t len_got,
              size_t len_expected, size_t rows, size_t cols, or_accuracy *acc);

/*
 * Acceptance check against the FP64 oracle rounded to half:
 *   masked entries (c >= valid, including pitch padding) are bit-exact 0x0000;
 *   unmasked entries within `ulp_tol` FP16 ulp or `abs_tol` absolute;
 *   |row sum - 1| <= rowsum_tol, summed in f64 over the FP16 outputs -- or,
 *   for a row whose FP64 oracle rounded to FP16 already misses rowsum_tol
 *   (FP16 rounding of many small probabilities), at most that row's oracle
 *   error plus floor_margin (floor_margin < 0: no such allowance); such rows
 *   are counted in floor_rows with the largest excess over the oracle.
 * `f64_ref` is the output of or_causal_softmax_f64_strided on the same input.
 */
typedef struct {
    int64_t checked_rows;
    int64_t mask_violations;
    int64_t elem_violations;
    int64_t rowsum_violations;
    int64_t first_bad_index; /* flat element index into the strided buffer, -1 if none */
    double max_abs;
    int64_t max_ulp;
    double max_rowsum_err;        /* of the checked output */
    double oracle_max_rowsum_err; /* of the FP64 oracle's own FP16 output */
    int64_t floor_rows;           /* rows accepted through the oracle's own row-sum error */
    double max_floor_excess;      /* their largest |sum - 1| above the oracle's */
} or_accept_report;

int or_accept_strided(const uint16_t *got, const uint16_t *f64_ref, int64_t batch,
                      int64_t batch_stride, int64_t rows, int64_t cols, int64_t pitch,
                      int64_t row_offset, double abs_tol, int64_t ulp_tol, double rowsum_tol,
                      double floor_margin, or_accept_report *report);

/*
 * Seeded synthetic score matrices of the benchmark workloads (the reference
 * publishes no dataset; these stand in for it). Restated here so the bench's
 * CPU leg and the tests can build inputs without the product library; the
 * tests check it bit for bit against the library's cs_generate.
 *   element (matrix b, absolute row r, column c): h = splitmix64(key(seed, b, r) + c),
 *   key(seed, b, r) = splitmix64(splitmix64(seed + K*b) + r);
 *   config 1: half(N(0,1)*4); 2: half(U(-8,8)); 3: half(N(0,1)*8) with 1% of entries
 *   +-60000 and two planted copies of each row's causal maximum; 4: half(N(0,1)*3);
 *   5: half(N(0,1)*2 + 0.001*c). N(0,1) by Box-Muller on 24-bit uniforms.
 * Pitch padding is written 0. Rows are split over `threads` POSIX threads.
 */
int or_generate(uint16_t *out, int config, uint64_t seed, int64_t batch, int64_t batch_stride,
                int64_t rows, int64_t cols, int64_t pitch, int64_t first_batch,
                int64_t first_row, int threads);

#ifdef __cplusplus
}
#endif

#endif /* CS_ORACLE_H */
