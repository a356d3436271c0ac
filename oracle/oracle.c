/*
 * CPU oracle for the fused causal softmax — TEST INFRASTRUCTURE ONLY.
 *
 * A C restatement of the reference project's CPU specification. Each function
 * names the reference file:line it follows. Build flags (oracle/Makefile) keep
 * IEEE single arithmetic exactly as the reference's Rust code performs it:
 * SSE2 floats, no FMA contraction, no fast-math, glibc expf (Rust's f32::exp
 * calls the platform libm expf on Linux).
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32, reference/src/lib.rs:30-83              */
/* ------------------------------------------------------------------ */

static inline uint32_t f32_bits(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    return b;
}

static inline float bits_f32(uint32_t b) {
    float x;
    memcpy(&x, &b, 4);
    return x;
}

/* reference/src/lib.rs:30-45: exact, including subnormals, infinities, NaNs. */
float or_half_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 31u;
    uint32_t frac = (uint32_t)h & 1023u;
    uint32_t bits;
    if (exp == 0 && frac == 0) {
        bits = sign;
    } else if (exp == 0) {
        /* Subnormal half: normalise the 10-bit fraction into an f32 normal. */
        uint32_t shift = (uint32_t)__builtin_clz(frac) - 21u;
        uint32_t mant = frac << shift;
        bits = sign | ((113u - shift) << 23) | ((mant & 1023u) << 13);
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (frac << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (frac << 13);
    }
    return bits_f32(bits);
}

/* reference/src/lib.rs:48-83: round-to-nearest-even, subnormals, overflow to inf.
 * f32 subnormals are below the half range and become signed zero. */
uint16_t or_f32_to_half(float x) {
    uint32_t bits = f32_bits(x);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exp = (int32_t)((bits >> 23) & 255u);
    uint32_t mant = bits & 0x7fffffu;
    if (exp == 255) return (uint16_t)(sign | (mant == 0 ? 0x7c00u : 0x7e00u));
    if (exp == 0) return sign;
    int32_t e = exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t v = mant | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t mask = (1u << shift) - 1u;
        uint32_t halfway = 1u << (shift - 1u);
        uint32_t r = v >> shift;
        uint32_t rem = v & mask;
        if (rem > halfway || (rem == halfway && (r & 1u))) r += 1u;
        return (uint16_t)(sign | r);
    }
    uint32_t m = mant >> 13;
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) m += 1u;
    return (uint16_t)(sign | (uint16_t)(((uint32_t)e << 10) + m));
}

/* Round a double to the nearest half, ties to even (for the FP64 oracle).
 * Scaling by a power of two is exact, so rint() (default FE_TONEAREST mode)
 * performs the single rounding step. */
uint16_t or_f64_to_half(double x) {
    uint16_t sign = signbit(x) ? 0x8000u : 0u;
    if (isnan(x)) return 0x7e00u;
    double a = fabs(x);
    if (a >= 65520.0) return (uint16_t)(sign | 0x7c00u); /* >= midpoint(65504, 65536) */
    if (a < 0x1p-14) {
        double q = rint(a * 0x1p24); /* units of the smallest subnormal */
        return (uint16_t)(sign | (uint16_t)q);
    }
    int k;
    (void)frexp(a, &k); /* a = f * 2^k, f in [0.5, 1) */
    int e = k - 1;      /* a = 1.m * 2^e, e in [-14, 15] */
    double r = rint(ldexp(a, 10 - e));
    if (r >= 2048.0) {
        r = 1024.0;
        e += 1;
    }
    if (e + 15 >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | (uint16_t)(((e + 15) << 10) + ((int)r - 1024)));
}

/* ------------------------------------------------------------------ */
/* Validation and padding, reference/src/lib.rs:110-152                */
/* ------------------------------------------------------------------ */

int or_validate(const uint16_t *scores, size_t len, size_t rows, size_t cols, float scale) {
    if (rows == 0 || cols == 0) return OR_EMPTY;
    size_t n;
    if (__builtin_mul_overflow(rows, cols, &n) || n != len) return OR_WRONG_LENGTH;
    if (!isfinite(scale) || !(scale >= 0.0f && scale <= OR_MAX_SCALE)) return OR_BAD_SCALE;
    for (size_t i = 0; i < len; ++i) {
        if (!isfinite(or_half_to_f32(scores[i]))) return OR_NON_FINITE;
    }
    return OR_OK;
}

size_t or_padded_pitch(size_t cols) { return (cols + 7u) & ~(size_t)7u; }

void or_pad(const uint16_t *scores, size_t rows, size_t cols, uint16_t *out) {
    size_t pitch = or_padded_pitch(cols);
    memset(out, 0, rows * pitch * sizeof(uint16_t));
    for (size_t r = 0; r < rows; ++r)
        memcpy(out + r * pitch, scores + r * cols, cols * sizeof(uint16_t));
}

void or_unpad(const uint16_t *padded, size_t rows, size_t cols, uint16_t *out) {
    size_t pitch = or_padded_pitch(cols);
    for (size_t r = 0; r < rows; ++r)
        memcpy(out + r * cols, padded + r * pitch, cols * sizeof(uint16_t));
}

/* ------------------------------------------------------------------ */
/* The f32 specification, reference/src/lib.rs:85-108                  */
/* ------------------------------------------------------------------ */

/* One row exactly as reference/src/lib.rs:93-106 computes it:
 *   max   = fold(-inf, f32::max) of half(x)*scale over c < valid,
 *   denom = sequential f32 sum of expf(half(x)*scale - max),
 *   out   = f32_to_half(expf(half(x)*scale - max) / denom) for c < valid,
 * and zero for every other column of the output row (width `out_width`). */
static void spec_row_f32(const uint16_t *x, uint16_t *y, int64_t valid, int64_t out_width,
                         float scale) {
    float max = -INFINITY;
    for (int64_t c = 0; c < valid; ++c) {
        float z = or_half_to_f32(x[c]) * scale;
        max = (z > max) ? z : max; /* f32::max; inputs are never NaN */
    }
    float denom = 0.0f;
    for (int64_t c = 0; c < valid; ++c) denom += expf(or_half_to_f32(x[c]) * scale - max);
    for (int64_t c = 0; c < valid; ++c) {
        float p = expf(or_half_to_f32(x[c]) * scale - max) / denom;
        y[c] = or_f32_to_half(p);
    }
    for (int64_t c = valid; c < out_width; ++c) y[c] = 0;
}

int or_causal_softmax(const uint16_t *scores, size_t len, size_t rows, size_t cols,
                      float scale, uint16_t *out) {
    int err = or_validate(scores, len, rows, cols, scale);
    if (err) return err;
    for (size_t r = 0; r < rows; ++r) {
        int64_t valid = (int64_t)((r + 1) < cols ? (r + 1) : cols);
        spec_row_f32(scores + r * cols, out + r * cols, valid, (int64_t)cols, scale);
    }
    return OR_OK;
}

/* FP64 restatement (reference/src/lib.rs:279-300): scale applied in double,
 * exp/sum/divide in double, the result rounded once to half. */
static void spec_row_f64(const uint16_t *x, uint16_t *y, int64_t valid, int64_t out_width,
                         float scale) {
    double s = (double)scale;
    double max = -INFINITY;
    for (int64_t c = 0; c < valid; ++c) {
        double z = (double)or_half_to_f32(x[c]) * s;
        if (z > max) max = z;
    }
    double denom = 0.0;
    for (int64_t c = 0; c < valid; ++c) denom += exp((double)or_half_to_f32(x[c]) * s - max);
    for (int64_t c = 0; c < valid; ++c)
        y[c] = or_f64_to_half(exp((double)or_half_to_f32(x[c]) * s - max) / denom);
    for (int64_t c = valid; c < out_width; ++c) y[c] = 0;
}

/* ------------------------------------------------------------------ */
/* Online-kernel arithmetic model, reference/src/online.rs:5-61         */
/* ------------------------------------------------------------------ */

/* reference/src/online.rs:5-17: 32-lane XOR butterfly, offsets 16..1. */
void or_butterfly(const float in[32], int maximum, float out[32]) {
    float lanes[32], before[32];
    memcpy(lanes, in, sizeof lanes);
    static const int offsets[5] = {16, 8, 4, 2, 1};
    for (int k = 0; k < 5; ++k) {
        memcpy(before, lanes, sizeof before);
        for (int lane = 0; lane < 32; ++lane) {
            float a = before[lane], b = before[lane ^ offsets[k]];
            lanes[lane] = maximum ? ((b > a) ? b : a) : (a + b);
        }
    }
    memcpy(out, lanes, sizeof lanes);
}

/* reference/src/online.rs:19-61: 128-column tiles, lane l owns columns
 * col0 + l + 32*item, online (max, denominator) recurrence per tile. */
int or_tiled_online_softmax(const uint16_t *scores, size_t len, size_t rows, size_t cols,
                            float scale, uint16_t *out) {
    int err = or_validate(scores, len, rows, cols, scale);
    if (err) return err;
    memset(out, 0, len * sizeof(uint16_t));
    for (size_t row = 0; row < rows; ++row) {
        size_t valid = (row + 1) < cols ? (row + 1) : cols;
        float maximum = -INFINITY, denominator = 0.0f;
        for (size_t col0 = 0; col0 < valid; col0 += 128) {
            float lanes[32][4], lane_max[32], red[32];
            for (int lane = 0; lane < 32; ++lane) {
                lane_max[lane] = -INFINITY;
                for (int item = 0; item < 4; ++item) {
                    size_t col = col0 + (size_t)lane + (size_t)item * 32;
                    float score = -INFINITY;
                    if (col < valid) score = or_half_to_f32(scores[row * cols + col]) * scale;
                    lanes[lane][item] = score;
                    if (score > lane_max[lane]) lane_max[lane] = score;
                }
            }
            or_butterfly(lane_max, 1, red);
            float next = (red[0] > maximum) ? red[0] : maximum;
            float lane_exp[32];
            for (int lane = 0; lane < 32; ++lane) {
                float e0 = expf(lanes[lane][0] - next);
                float e1 = expf(lanes[lane][1] - next);
                float e2 = expf(lanes[lane][2] - next);
                float e3 = expf(lanes[lane][3] - next);
                lane_exp[lane] = (e0 + e1) + (e2 + e3);
            }
            or_butterfly(lane_exp, 0, red);
            denominator = denominator * expf(maximum - next) + red[0];
            maximum = next;
        }
        for (size_t col = 0; col < valid; ++col) {
            float score = or_half_to_f32(scores[row * cols + col]) * scale;
            out[row * cols + col] = or_f32_to_half(expf(score - maximum) / denominator);
        }
    }
    return OR_OK;
}

/* ------------------------------------------------------------------ */
/* Strided / batched / row-offset drivers (threaded over rows)          */
/* ------------------------------------------------------------------ */

typedef struct {
    const uint16_t *in;
    uint16_t *out;
    int64_t batch_stride, rows, cols, pitch, row_offset;
    float scale;
    int64_t begin, end; /* flat (matrix * rows + row) range */
    int f64;
} strided_job;

static void *strided_worker(void *arg) {
    const strided_job *j = (const strided_job *)arg;
    for (int64_t t = j->begin; t < j->end; ++t) {
        int64_t b = t / j->rows, i = t % j->rows;
        int64_t abs_row = j->row_offset + i;
        int64_t valid = (abs_row + 1) < j->cols ? (abs_row + 1) : j->cols;
        const uint16_t *x = j->in + b * j->batch_stride + i * j->pitch;
        uint16_t *y = j->out + b * j->batch_stride + i * j->pitch;
        if (j->f64)
            spec_row_f64(x, y, valid, j->pitch, j->scale);
        else
            spec_row_f32(x, y, valid, j->pitch, j->scale);
    }
    return NULL;
}

static int run_strided(const uint16_t *in, uint16_t *out, int64_t batch, int64_t batch_stride,
                       int64_t rows, int64_t cols, int64_t pitch, int64_t row_offset,
                       float scale, int threads, int f64) {
    if (batch <= 0 || rows <= 0 || cols <= 0) return OR_EMPTY;
    if (pitch < cols || row_offset < 0 || (batch > 1 && batch_stride < rows * pitch))
        return OR_WRONG_LENGTH;
    if (!isfinite(scale) || !(scale >= 0.0f && scale <= OR_MAX_SCALE)) return OR_BAD_SCALE;
    int64_t total = batch * rows;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((int64_t)threads > total) threads = (int)total;
    strided_job jobs[256];
    pthread_t tids[256];
    int64_t per = (total + threads - 1) / threads;
    for (int k = 0; k < threads; ++k) {
        jobs[k] = (strided_job){in, out, batch_stride, rows, cols, pitch, row_offset, scale,
                                (int64_t)k * per, ((int64_t)k + 1) * per, f64};
        if (jobs[k].end > total) jobs[k].end = total;
    }
    if (threads == 1) {
        strided_worker(&jobs[0]);
        return OR_OK;
    }
    int started = 0;
    for (int k = 0; k < threads; ++k) {
        if (pthread_create(&tids[k], NULL, strided_worker, &jobs[k]) != 0) {
            strided_worker(&jobs[k]); /* run inline if a thread cannot start */
            tids[k] = 0;
        } else {
            ++started;
        }
    }
    for (int k = 0; k < threads; ++k)
        if (tids[k]) pthread_join(tids[k], NULL);
    (void)started;
    return OR_OK;
}

int or_causal_softmax_strided(const uint16_t *in, uint16_t *out, int64_t batch,
                              int64_t batch_stride, int64_t rows, int64_t cols,
                              int64_t pitch, int64_t row_offset, float scale, int threads) {
    return run_strided(in, out, batch, batch_stride, rows, cols, pitch, row_offset, scale,
                       threads, 0);
}

int or_causal_softmax_f64_strided(const uint16_t *in, uint16_t *out, int64_t batch,
                                  int64_t batch_stride, int64_t rows, int64_t cols,
                                  int64_t pitch, int64_t row_offset, float scale, int threads) {
    return run_strided(in, out, batch, batch_stride, rows, cols, pitch, row_offset, scale,
                       threads, 1);
}

/* ------------------------------------------------------------------ */
/* Verifier, host/src/lib.rs:280-328                                    */
/* ------------------------------------------------------------------ */

int or_verify(const uint16_t *got, const uint16_t *expected, size_t len_got,
              size_t len_expected, size_t rows, size_t cols, or_accuracy *acc) {
    or_accuracy m = {0.0f, 0.0f, 0.0f, -1, 0.0f, 0.0f};
    size_t n;
    if (len_got != len_expected || __builtin_mul_overflow(rows, cols, &n) || n != len_got) {
        if (acc) *acc = m;
        return OR_VERIFY_LENGTH;
    }
    int code = OR_VERIFY_OK;
    for (size_t row = 0; row < rows && code == OR_VERIFY_OK; ++row) {
        float sum = 0.0f;
        for (size_t col = 0; col < cols; ++col) {
            size_t i = row * cols + col;
            float g = or_half_to_f32(got[i]), w = or_half_to_f32(expected[i]);
            if (!isfinite(g)) { code = OR_VERIFY_NON_FINITE; m.index = (int64_t)i; break; }
            if (g < 0.0f) { code = OR_VERIFY_NEGATIVE; m.index = (int64_t)i; break; }
            if (col > row && got[i] != 0) { code = OR_VERIFY_MASK; m.index = (int64_t)i; break; }
            float err = fabsf(g - w);
            if (err > m.max_abs) m.max_abs = err;
            if (w > 0.0001f && err / w > m.max_relative) m.max_relative = err / w;
            if (err > 0.003f + 0.003f * fabsf(w)) {
                code = OR_VERIFY_ELEMENT;
                m.index = (int64_t)i;
                m.got = g;
                m.want = w;
                break;
            }
            sum += g;
        }
        if (code != OR_VERIFY_OK) break;
        float rs = fabsf(sum - 1.0f);
        if (rs > m.max_row_sum_error) m.max_row_sum_error = rs;
        if (rs > 0.02f) {
            code = OR_VERIFY_ROW_SUM;
            m.index = (int64_t)row;
            m.got = sum;
        }
    }
    if (acc) *acc = m;
    return code;
}

/* ------------------------------------------------------------------ */
/* Acceptance against the FP64 oracle                                   */
/* ------------------------------------------------------------------ */

int or_accept_strided(const uint16_t *got, const uint16_t *f64_ref, int64_t batch,
                      int64_t batch_stride, int64_t rows, int64_t cols, int64_t pitch,
                      int64_t row_offset, double abs_tol, int64_t ulp_tol, double rowsum_tol,
                      double floor_margin, or_accept_report *report) {
    or_accept_report r;
    memset(&r, 0, sizeof r);
    r.first_bad_index = -1;
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t i = 0; i < rows; ++i) {
            int64_t abs_row = row_offset + i;
            int64_t valid = (abs_row + 1) < cols ? (abs_row + 1) : cols;
            int64_t base = b * batch_stride + i * pitch;
            double sum = 0.0, ref_sum = 0.0;
            for (int64_t c = 0; c < pitch; ++c) {
                uint16_t g = got[base + c];
                if (c >= valid) {
                    if (g != 0) {
                        if (r.first_bad_index < 0) r.first_bad_index = base + c;
                        r.mask_violations++;
                    }
                    continue;
                }
                uint16_t w = f64_ref[base + c];
                float gf = or_half_to_f32(g), wf = or_half_to_f32(w);
                sum += (double)gf;
                ref_sum += (double)wf;
                int bad = !isfinite(gf) || (g & 0x8000u);
                double ad = fabs((double)gf - (double)wf);
                int64_t ulp = (int64_t)g > (int64_t)w ? (int64_t)g - w : (int64_t)w - g;
                if (!bad && ad > r.max_abs) r.max_abs = ad;
                if (!bad && ulp > r.max_ulp) r.max_ulp = ulp;
                if (bad || (ulp > ulp_tol && ad > abs_tol)) {
                    if (r.first_bad_index < 0) r.first_bad_index = base + c;
                    r.elem_violations++;
                }
            }
            double e = fabs(sum - 1.0), oe = fabs(ref_sum - 1.0);
            if (e > r.max_rowsum_err) r.max_rowsum_err = e;
            if (oe > r.oracle_max_rowsum_err) r.oracle_max_rowsum_err = oe;
            /* A row whose exactly rounded (FP64 -> FP16) values already miss
             * rowsum_tol may miss it by as much, plus floor_margin (< 0: no
             * such allowance). */
            int ok = e <= rowsum_tol;
            if (!ok && floor_margin >= 0.0 && oe > rowsum_tol && e <= oe + floor_margin) {
                ok = 1;
                r.floor_rows++;
                if (e - oe > r.max_floor_excess) r.max_floor_excess = e - oe;
            }
            if (!ok) {
                if (r.first_bad_index < 0) r.first_bad_index = base;
                r.rowsum_violations++;
            }
            r.checked_rows++;
        }
    }
    if (report) *report = r;
    return (r.mask_violations || r.elem_violations || r.rowsum_violations) ? 1 : 0;
}

/* ------------------------------------------------------------------ */
/* Benchmark workload generator (synthetic stand-in for a dataset)      */
/* ------------------------------------------------------------------ */

/* Vigna's splitmix64 finaliser (public-domain published algorithm). */
static inline uint64_t gen_mix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* Box-Muller on two 24-bit uniforms of one hash; the first is in (0, 1]. */
static inline double gen_normal(uint64_t h) {
    const double u1 = (double)((h >> 40) + 1) * (1.0 / 16777216.0);
    const double u2 = (double)((h >> 16) & 0xFFFFFFu) * (1.0 / 16777216.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

typedef struct {
    uint16_t *out;
    int config;
    uint64_t seed;
    int64_t stride, rows, cols, pitch, first_batch, first_row, begin, end;
} gen_job;

static void *gen_worker(void *arg) {
    const gen_job *j = (const gen_job *)arg;
    for (int64_t t = j->begin; t < j->end; ++t) {
        const int64_t b = t / j->rows, r = t % j->rows, a = j->first_row + r;
        uint16_t *y = j->out + b * j->stride + r * j->pitch;
        const uint64_t key =
            gen_mix(gen_mix(j->seed + 0x632BE59BD9B4E019ull * (uint64_t)(j->first_batch + b)) + (uint64_t)a);
        for (int64_t c = 0; c < j->cols; ++c) {
            const uint64_t h = gen_mix(key + (uint64_t)c);
            double v;
            if (j->config == 1) {
                v = gen_normal(h) * 4.0;
            } else if (j->config == 2) {
                v = -8.0 + 16.0 * ((double)(h >> 11) * (1.0 / 9007199254740992.0));
            } else if (j->config == 3) {
                const uint64_t h2 = gen_mix(h ^ 0xD1B54A32D192ED03ull);
                v = (h2 % 100 == 0) ? (((h2 >> 32) & 1u) ? 60000.0 : -60000.0) : gen_normal(h) * 8.0;
            } else if (j->config == 4) {
                v = gen_normal(h) * 3.0;
            } else {
                v = gen_normal(h) * 2.0 + 0.001 * (double)c;
            }
            y[c] = or_f32_to_half((float)v);
        }
        for (int64_t c = j->cols; c < j->pitch; ++c) y[c] = 0;
        if (j->config == 3 && a >= 1) {
            /* Two more copies of the row's causal maximum at distinct columns. */
            const int64_t valid = (a + 1) < j->cols ? (a + 1) : j->cols;
            if (valid >= 2) {
                int64_t arg = 0;
                float best = or_half_to_f32(y[0]);
                for (int64_t c = 1; c < valid; ++c) {
                    const float f = or_half_to_f32(y[c]);
                    if (f > best) {
                        best = f;
                        arg = c;
                    }
                }
                const uint16_t mbits = y[arg];
                const uint64_t hk = gen_mix(key ^ 0x8CB92BA72F3D8DD7ull);
                const int64_t c1 = (int64_t)(hk % (uint64_t)valid);
                const int64_t c2 = (c1 + 1 + (int64_t)((hk >> 32) % (uint64_t)(valid - 1))) % valid;
                y[c1] = mbits;
                y[c2] = mbits;
            }
        }
    }
    return NULL;
}

int or_generate(uint16_t *out, int config, uint64_t seed, int64_t batch, int64_t batch_stride,
                int64_t rows, int64_t cols, int64_t pitch, int64_t first_batch,
                int64_t first_row, int threads) {
    if (!out || config < 1 || config > 5) return OR_WRONG_LENGTH;
    if (batch <= 0 || rows <= 0 || cols <= 0) return OR_EMPTY;
    if (pitch < cols || first_row < 0 || first_batch < 0) return OR_WRONG_LENGTH;
    if (batch > 1 && batch_stride < rows * pitch) return OR_WRONG_LENGTH;
    const int64_t total = batch * rows;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((int64_t)threads > total) threads = (int)total;
    gen_job jobs[256];
    pthread_t tids[256];
    const int64_t per = (total + threads - 1) / threads;
    for (int k = 0; k < threads; ++k) {
        jobs[k] = (gen_job){out, config, seed, batch > 1 ? batch_stride : rows * pitch, rows, cols,
                            pitch, first_batch, first_row, (int64_t)k * per,
                            ((int64_t)k + 1) * per < total ? ((int64_t)k + 1) * per : total};
        tids[k] = 0;
    }
    if (threads == 1) {
        gen_worker(&jobs[0]);
        return OR_OK;
    }
    for (int k = 0; k < threads; ++k)
        if (pthread_create(&tids[k], NULL, gen_worker, &jobs[k]) != 0) {
            gen_worker(&jobs[k]); /* run inline if a thread cannot start */
            tids[k] = 0;
        }
    for (int k = 0; k < threads; ++k)
        if (tids[k]) pthread_join(tids[k], NULL);
    return OR_OK;
}
