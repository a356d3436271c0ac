/*
 * causal_softmax.h — C ABI of the B200 (sm_100a) fused causal softmax.
 *
 *   P[r,c] = exp(scale*S[r,c] - max_r) / sum_{j<=r} exp(scale*S[r,j] - max_r)   for c <= r
 *   P[r,c] = +0.0 (bit pattern 0x0000)                                         otherwise
 *
 * S and P are IEEE binary16 stored as uint16_t bits, row-major with a row
 * pitch (elements) that is a multiple of 8, so every row starts 16-byte
 * aligned; arithmetic is binary32. The masked upper triangle is never read,
 * and every output column the softmax does not own — including the pitch
 * padding — is written 0x0000.
 *
 * Every entry point stands in for a piece of the reference project's host
 * surface (R-P-Padhi/GB200-SM100A-TMA-Fused-Causal-Attention-Softmax; file:line
 * citations below are paths inside that project). Plain pointers and sizes
 * only: device pointers are CUDA device addresses, `stream` is a
 * cudaStream_t passed as void*. Functions return 0 (CS_OK) or a negative
 * CS_ERR_* code; none of them allocates or frees caller buffers.
 *
 * Threads: distinct plans and sessions may be used from different host
 * threads concurrently; one plan or session must not be used by two threads
 * at once.
 */
#ifndef CAUSAL_SOFTMAX_H
#define CAUSAL_SOFTMAX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CS_ABI_VERSION 1

/* Kernel selection. Mirrors host/src/lib.rs:5-13 (enum Kernel) and the names
 * host/src/lib.rs:22-42 parses; each name selects this library's design:
 *   BASELINE : one CTA per row, three passes over global memory (control)
 *   WARP     : narrow rows, one 16-byte vector per lane (cols <= 32)
 *   TMA      : row-resident single pass, TMA bulk-copy ring, thread stores
 *   PIPELINE : as TMA, with TMA bulk stores of the output
 *   ONLINE   : pipelined online-softmax over 8 KB tiles for long rows
 *   AUTO     : resolved by cs_resolve_kernel */
typedef enum cs_kernel {
    CS_KERNEL_AUTO = 0,
    CS_KERNEL_BASELINE = 1,
    CS_KERNEL_WARP = 2,
    CS_KERNEL_TMA = 3,
    CS_KERNEL_PIPELINE = 4,
    CS_KERNEL_ONLINE = 5
} cs_kernel;

/* Error codes. -1..-4 mirror reference/src/lib.rs:8-27 (ShapeError); the
 * warp-width error mirrors gpu/src/driver.rs:149-151; the alignment/pitch
 * errors mirror the tensor_map checks gpu/src/main.rs:737-742; the size
 * limits mirror host/src/lib.rs:143-168 (Config::validate). */
enum {
    CS_OK = 0,
    CS_ERR_EMPTY = -1,          /* matrix dimensions must be positive */
    CS_ERR_WRONG_LENGTH = -2,   /* sizes overflow or buffer/stride too small */
    CS_ERR_BAD_SCALE = -3,      /* scale must be finite and in [0, 1e30] */
    CS_ERR_NON_FINITE = -4,     /* score matrix contains NaN or infinity */
    CS_ERR_WARP_COLS = -5,      /* warp specialization requires cols <= 32 */
    CS_ERR_ALIGNMENT = -6,      /* base pointer not 16-byte aligned */
    CS_ERR_PITCH = -7,          /* pitch < cols, not a multiple of 8, or too large */
    CS_ERR_BAD_KERNEL = -8,     /* unknown kernel */
    CS_ERR_DEVICE = -9,         /* no usable sm_100 device */
    CS_ERR_CUDA = -10,          /* a CUDA runtime call failed */
    CS_ERR_TIMEOUT = -11,       /* a bounded device-side wait ran out */
    CS_ERR_NULL = -12,          /* null pointer argument */
    CS_ERR_PADDING = -13,       /* nonzero padded output found */
    CS_ERR_UNSUPPORTED = -14,   /* shape beyond the selected kernel's limits */
    CS_ERR_PROBE = -15,         /* probe kernel returned a wrong value */
    CS_ERR_ARG = -16,           /* other invalid argument */
    CS_ERR_STATUS = -17         /* device status word holds bits no kernel defines */
};

#define CS_MAX_SCALE 1.0e30f   /* reference/src/lib.rs:5 */

/* Device status word bits reported by cs_plan_status (and the session and
 * no-alloc status reads). A kernel sets only CS_STATUS_TIMEOUT: a bounded
 * device-side wait ran out. Every other bit is reserved. */
#define CS_STATUS_TIMEOUT 1u

/* ---------------------------------------------------------------- */
/* Host-only queries (no GPU needed)                                 */
/* ---------------------------------------------------------------- */

int cs_abi_version(void);

/* Static message for a CS_* code; never NULL. */
const char *cs_strerror(int code);

/* Detail of the last error raised on the calling thread (CUDA error text,
 * offending size); empty if none. Thread-local storage, never NULL. */
const char *cs_last_error_detail(void);

/* host/src/lib.rs:22-31 (Kernel::name). NULL for an unknown value. */
const char *cs_kernel_name(int kernel);

/* host/src/lib.rs:32-42 (Kernel::parse). Returns the cs_kernel value or CS_ERR_BAD_KERNEL. */
int cs_kernel_parse(const char *name);

/* host/src/lib.rs:43-45 (Kernel::supports): 1 if `kernel` accepts `cols`, else 0. */
int cs_kernel_supports(int kernel, int64_t cols);

/* host/src/lib.rs:169-177 (Config::resolved_kernel) for this library:
 * WARP for cols <= 32, PIPELINE while a row pair (else a row) fits the row-resident kernel,
 * ONLINE beyond. Non-AUTO values are returned unchanged. Decides for whole
 * matrices (row offset 0), like the reference; a plan for a row block decides
 * with its own offset, so a block of long rows may resolve to ONLINE where
 * this returns PIPELINE. */
int cs_resolve_kernel(int kernel, int64_t rows, int64_t cols);

/* host/src/lib.rs:49-64 (Kernel::logical_bytes) for this library's kernels:
 * modelled HBM bytes of one matrix (read traffic of each kernel + one write
 * of the full rows x cols output). Returns a negative value for AUTO or an
 * unknown kernel. */
double cs_logical_bytes(int kernel, int64_t rows, int64_t cols);

/* Algorithmic bytes of one matrix: 2*T + 2*rows*cols, T = causal element
 * count of rows [row_offset, row_offset+rows) (host/src/lib.rs:52-56 for
 * row_offset 0). The roofline every kernel is measured against. */
double cs_roofline_bytes(int64_t rows, int64_t cols, int64_t row_offset);

/* reference/src/lib.rs:132-134: pitch = round_up(cols, 8). */
int64_t cs_padded_pitch(int64_t cols);

/* Argument checks every launch performs (reference/src/lib.rs:110-129 for
 * shape and scale, host/src/lib.rs:143-168 for the size limits,
 * gpu/src/main.rs:737-742 for the pitch rule). batch_stride is ignored when
 * batch == 1. Does not inspect data (see cs_check_finite_host). */
int cs_validate(int64_t batch, int64_t batch_stride, int64_t rows, int64_t cols, int64_t pitch,
                int64_t row_offset, float scale);

/* reference/src/lib.rs:125-127: CS_ERR_NON_FINITE if any of `n` halves is
 * NaN or infinite, else CS_OK. */
int cs_check_finite_host(const uint16_t *scores, int64_t n);

/* The error code a device status word maps to, as every status read in this
 * library reports it (the reference propagates device failures as errors,
 * gpu/src/driver.rs:108-211): CS_OK for 0, CS_ERR_TIMEOUT when
 * CS_STATUS_TIMEOUT is set, CS_ERR_STATUS for any other (reserved) bit. */
int cs_status_error(uint32_t status);

/* ---------------------------------------------------------------- */
/* Device path: plans (replaces gpu/src/driver.rs:65-211)            */
/* ---------------------------------------------------------------- */

typedef struct cs_plan cs_plan;

/* Describe a launch target once: `batch` matrices at d_in/d_out (element
 * stride batch_stride between matrices), each `rows` x `cols` with row pitch
 * `pitch`; local row i is absolute causal row row_offset + i (row-block
 * shards). Replaces Session::prepare_on + tensor_map (gpu/src/driver.rs:65-95,
 * gpu/src/main.rs:730-774): the plan keeps the launch geometry and a 256-byte
 * device status word (the only allocation it makes). The caller keeps
 * ownership of d_in/d_out, which may alias only if d_in == d_out is NOT used
 * (in-place is not supported). */
int cs_plan_create(cs_plan **plan, int device, const void *d_in, void *d_out, int64_t batch,
                   int64_t batch_stride, int32_t rows, int32_t cols, int32_t pitch,
                   int32_t row_offset);

/* Enqueue the softmax on `stream` (replaces Session::launch_on,
 * gpu/src/driver.rs:108-211). Asynchronous: no host synchronisation and no
 * allocation. Launches of one plan must not overlap on the GPU (issue them
 * on one stream, or order them with events): they share the plan's output
 * and the work-schedule counters in its device word block. Errors: argument errors as cs_validate, CS_ERR_WARP_COLS,
 * CS_ERR_UNSUPPORTED, CS_ERR_CUDA. */
int cs_plan_launch(cs_plan *plan, int kernel, float scale, void *stream);

/* Synchronise the plan's device and read (then clear) its status word.
 * *status receives the CS_STATUS_* bits; returns cs_status_error of them. */
int cs_plan_status(cs_plan *plan, uint32_t *status);

/* Bound, in nanoseconds of GPU time, on every device-side wait of later
 * launches of this plan (default 2 s). */
int cs_plan_set_timeout(cs_plan *plan, uint64_t timeout_ns);

/* Folded row-block shard (no counterpart in the reference, which has no
 * multi-GPU path; extends the row_offset of cs_plan_create): local rows
 * split_row..rows-1 of every matrix are absolute causal rows split_offset,
 * split_offset+1, ... — a second row block stored right after the first.
 * For an M-row causal matrix over N ranks, rank k holding block [a, b) and
 * its mirror [M-b, M-a) (split_row = b - a, split_offset = M - b) gets units
 * of M+1 causal elements each, as the whole matrix does, instead of a block
 * of only the longest rows. Needs 0 < split_row < rows and split_offset >=
 * row_offset + split_row (else CS_ERR_ARG); split_row = 0 restores one
 * contiguous block. Affects later launches of the plan. */
int cs_plan_set_row_split(cs_plan *plan, int32_t split_row, int32_t split_offset);

/* Tuning knobs (0 / -1 = automatic): vectors per thread of the TMA /
 * PIPELINE kernels (2, 4 or 8; 16 + i selects compiled variant i of the
 * row-resident kernel directly) or of the ONLINE kernel (0: automatic, which
 * is 160-thread CTAs with 4 KB tiles for rows of up to 8192 columns and the
 * shape of 2 beyond; 2: 288-thread CTAs, 8 consumer warps with 8 KB tiles;
 * 1: 1024-thread CTAs, 31 consumer warps with 15.5 KB tiles; 3: each row held
 * whole in the shared memory of a cluster of 2 to 16 CTAs that exchange
 * their partial statistics through distributed shared memory; 2..8 rows in
 * flight per cluster), ring stages of the TMA / PIPELINE / ONLINE
 * kernels (1..32; fewer where shared memory does not hold them), L2
 * evict-first hint on the input copies (0 off, 1 on),
 * masked columns written by TMA bulk stores (1) or by thread stores (0). */
int cs_plan_set_tuning(cs_plan *plan, int vec_per_thread, int stages, int l2_hint,
                       int zero_fill_tma);

/* TMA / PIPELINE kernels: the input rows of the first `prefetch_units` work
 * units of each CTA (row pairs; -1 = automatic, 0..1024, never fewer than
 * the ring's first stages) are pulled into L2 while the previous kernel in
 * the stream is still finishing, before the launch waits for it (a
 * prefetch consumes no data). Affects later launches of the plan; one-shot
 * launches (cs_softmax*) use the automatic depth. */
int cs_plan_set_prefetch(cs_plan *plan, int prefetch_units);

typedef struct cs_launch_info {
    int32_t kernel;          /* resolved cs_kernel */
    int32_t grid;            /* CTAs per launch */
    int32_t block;           /* threads per CTA */
    int32_t smem_bytes;      /* dynamic shared memory per CTA */
    int32_t stages;          /* ring depth (TMA/PIPELINE/ONLINE), else 0 */
    int32_t vec_per_thread;  /* TMA/PIPELINE registers: 16-byte vectors per thread */
    int32_t ctas_per_sm;     /* resident CTAs per SM from the occupancy query */
    int32_t launches;        /* kernel launches per cs_plan_launch (always 1) */
    int64_t units;           /* work units (row pairs, rows) per launch */
    double algorithmic_bytes;/* roofline bytes per launch (all matrices) */
    double modelled_bytes;   /* the kernel's own modelled HBM bytes per launch */
} cs_launch_info;

/* Launch geometry a cs_plan_launch with `kernel` would use. */
int cs_plan_describe(cs_plan *plan, int kernel, cs_launch_info *info);

/* Test hook: launch with debug flags (1 = the producer issues no copies, so
 * every consumer wait must run out after `timeout_ns` and report
 * CS_STATUS_TIMEOUT). Not for production use. */
int cs_plan_launch_debug(cs_plan *plan, int kernel, float scale, void *stream, uint32_t flags,
                         uint64_t timeout_ns);

void cs_plan_destroy(cs_plan *plan);

/* One-shot launches on the current device (no plan object). The status word
 * is a per-device buffer the library allocates on the first call for that
 * device. cs_softmax has the argument meaning of the reference's kernel
 * launches (gpu/src/main.rs:72-78: input, output, cols, pitch, scale). */
int cs_softmax(int kernel, const void *d_in, void *d_out, int32_t rows, int32_t cols,
               int32_t pitch, float scale, void *stream);

int cs_softmax_batched(int kernel, const void *d_in, void *d_out, int64_t batch,
                       int64_t batch_stride, int32_t rows, int32_t cols, int32_t pitch,
                       int32_t row_offset, float scale, void *stream);

/* No counterpart in the reference. cs_softmax_batched with the same arguments
 * and results, for callers that may not allocate device memory: a serving
 * engine or framework whose caching allocator owns the GPU's memory and
 * budgets every byte, and which cannot let a library call cudaMalloc behind
 * its back (cudaMalloc can synchronize the device and takes memory outside
 * that budget). cs_softmax_batched allocates a 256-byte status word on its
 * first call on each device; this entry point allocates nothing. Its only
 * scratch is the kernels' status word, taken from a static device array of
 * CS_NOALLOC_SLOTS 32-bit words (256 bytes) in the library's device image,
 * which every GPU that loads the library holds until the process exits.
 *
 * `slot` picks the word (0 <= slot < CS_NOALLOC_SLOTS, else CS_ERR_ARG with a
 * message). The call clears that word on `stream` before the launch, since it
 * keeps the previous call's bits. Calls that overlap on the GPU and use the
 * same slot race on it: one call's clear can erase the other's timeout bit.
 * Callers that launch on several streams at once give each stream its own
 * slot. If `status` is non-null the call waits for `stream`, stores the
 * CS_STATUS_* bits there and returns cs_status_error of them; if it is null
 * the call returns after the launch, and the slot's word can be read later
 * with cs_noalloc_status.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, which may load the library's device code); make that
 * first call before any stream capture. Errors: as cs_softmax_batched, plus
 * CS_ERR_ARG for a bad slot. */
#define CS_NOALLOC_SLOTS 64
int cs_softmax_noalloc(int kernel, const void *d_in, void *d_out, int64_t batch,
                       int64_t batch_stride, int32_t rows, int32_t cols, int32_t pitch,
                       int32_t row_offset, float scale, int32_t slot, uint32_t *status,
                       void *stream);

/* No counterpart in the reference. Reads, then clears, the status word of
 * no-alloc slot `slot` on the current device, for callers that passed a null
 * `status` to cs_softmax_noalloc and synchronise on their own terms: the copy
 * and the clear are ordered on `stream` after the launches issued there, and
 * the call waits for `stream` before it stores the bits in *status. Allocates
 * nothing. Returns cs_status_error of the bits, CS_ERR_ARG for a bad slot,
 * CS_ERR_NULL for a null `status`. A later launch on the same slot clears the
 * word itself, so read it before reusing the slot. */
int cs_noalloc_status(int32_t slot, uint32_t *status, void *stream);

/* ---------------------------------------------------------------- */
/* Sessions: host buffers (replaces gpu/src/driver.rs:12-59, 213-248) */
/* ---------------------------------------------------------------- */

typedef struct cs_session cs_session;

/* Bind a device (requires compute capability 10.x, gpu/src/driver.rs:29-42)
 * and create the session's streams. */
int cs_session_create(cs_session **session, int device);

/* gpu/src/driver.rs:44-59: run the probe kernel (out[i] = i ^ 0x5a5a5a5a
 * over 256 lanes) and check every lane. CS_ERR_PROBE on a mismatch. */
int cs_session_probe(cs_session *session);

/* End to end from host memory: `batch` dense rows x cols matrices (no
 * padding, like reference/src/lib.rs:85) are copied to the device with the
 * padded pitch, softmaxed, and copied back unpadded into h_out. Local row i
 * is absolute causal row row_offset + i (0 for whole matrices). Only causal
 * bytes cross PCIe: rows travel in blocks of 256, each as wide as its widest
 * row (cs_host_copy_bytes gives the bytes per direction), and the rest of
 * each output row is written +0.0 by up to 8 host threads while the copies
 * run; the input's masked part is never read. Chunks of matrices alternate
 * between two streams so host->device copies, kernels and device->host
 * copies overlap; device buffers are cached in the session. Pinned host
 * memory (cs_host_register) makes the copies asynchronous. Returns after the
 * last copy has landed and the zeroing threads have finished; checks the
 * status word. */
int cs_session_softmax_host(cs_session *session, int kernel, const uint16_t *h_in,
                            uint16_t *h_out, int64_t batch, int32_t rows, int32_t cols,
                            int32_t row_offset, float scale);

/* The reference's prepare / launch / result cycle (gpu/src/driver.rs:65-95,
 * 108-211, 213-232) for one matrix: prepare copies `h_in` (dense rows x cols)
 * into a padded device buffer and fills the output with the 0xfb00
 * sentinel; launch runs `kernel`; result synchronises, checks that the
 * padding columns are zero (CS_ERR_PADDING) and copies the unpadded output
 * to h_out. */
int cs_session_prepare(cs_session *session, const uint16_t *h_in, int32_t rows, int32_t cols);
int cs_session_launch(cs_session *session, int kernel, float scale);
int cs_session_result(cs_session *session, uint16_t *h_out);

/* The session's primary stream (cudaStream_t as void*). */
void *cs_session_stream(cs_session *session);

/* Bytes cs_session_softmax_host moves in each direction for `batch`
 * rows x cols matrices starting at causal row row_offset (a host-only query;
 * the reference copies whole matrices, gpu/src/driver.rs:65-95, 213-232).
 * CS_ERR_EMPTY for non-positive sizes. */
int64_t cs_host_copy_bytes(int64_t batch, int32_t rows, int32_t cols, int32_t row_offset);

void cs_session_destroy(cs_session *session);

/* Page-lock / release caller host memory for asynchronous copies. */
int cs_host_register(void *ptr, size_t bytes);
int cs_host_unregister(void *ptr);

/* Number of SMs of `device` (for grid sizing by callers), or a CS_ERR_* code. */
int cs_device_sm_count(int device);

#ifdef __cplusplus
}
#endif

#endif /* CAUSAL_SOFTMAX_H */
