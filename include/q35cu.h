/*
 * q35cu.h -- the native API of libq35cuda.so beyond the reference's
 * q35_mm.h: device-resident weights, device-pointer launches on a caller
 * stream, error reporting, and the tensor-parallel (NCCL) primitives.
 *
 * The reference engine has no counterpart for most of this (it is a
 * single-process CPU library, qwen35-c/include/q35/q35_mm.h); each entry
 * below says which reference behaviour it extends.  Host-pointer callers
 * only ever need q35_mm.h.
 *
 * Conventions
 *   - every function returns a q35cu_status (0 = OK) unless stated;
 *   - the last failure of the calling thread is kept for q35cu_last_error();
 *   - "stream" is a cudaStream_t passed as void* (NULL = the library's own
 *     per-device stream);
 *   - activations are fp32 row-major, token-major: X [m, ldx], Y [m, ldy].
 */
#ifndef Q35CU_H
#define Q35CU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    Q35CU_OK = 0,
    Q35CU_ERR_ARG = 1,          /* null pointer, zero/oversized shape, bad stride */
    Q35CU_ERR_NOMEM = 2,        /* device allocation failed or the budget is spent */
    Q35CU_ERR_CUDA = 3,         /* CUDA runtime error (message has the name) */
    Q35CU_ERR_UNSUPPORTED = 4,  /* shape or alignment the requested kernel cannot take */
    Q35CU_ERR_NCCL = 5,         /* NCCL call failed, or tensor parallel not initialised */
    Q35CU_ERR_NODEV = 6,        /* no CUDA device / not an sm_100 part */
    Q35CU_ERR_TIMEOUT = 7       /* a bounded device-side wait gave up */
} q35cu_status;

typedef enum { Q35CU_ON_ERROR_ABORT = 0, Q35CU_ON_ERROR_RECORD = 1 } q35cu_error_mode;

/* ---- errors ------------------------------------------------------------ */
/* The reference's matmuls return void and have no error channel
 * (qwen35-c/src/q35_mm.c:144-198); these add one. */
int q35cu_last_error(void);
const char *q35cu_last_error_message(void);
void q35cu_clear_error(void);
/* ABORT (default; env Q35CU_ON_ERROR=record flips it): a failing q35_mm_*
 * call prints the error and aborts.  RECORD: it records the error, fills
 * the outputs with NaN and returns. */
void q35cu_set_error_mode(int mode);
int q35cu_get_error_mode(void);

/* ---- device and residency cache --------------------------------------- */
int q35cu_device_count(void);                 /* 0 without a usable GPU */
int q35cu_set_device(int device);             /* device for later calls of this process */
int q35cu_sm_count(void);
/* Bytes of weights held by the q35_mm_* residency cache. */
size_t q35cu_cache_bytes(void);
/* Cap on device bytes for uploads (0 = no cap).  An upload over the cap
 * fails with Q35CU_ERR_NOMEM exactly like a failed cudaMalloc. */
void q35cu_set_memory_budget(size_t bytes);
/* Drop every cached upload (the engine's model free, qwen35-c/src/q35_model.c:714-729,
 * unmaps the weights; call this before reusing the host memory). */
void q35cu_release_all(void);
/* Drop cached uploads whose host weight pointer is W; returns how many. */
int q35cu_forget(const void *W);

/* ---- device-resident weights ------------------------------------------ */
typedef struct q35cu_weight q35cu_weight;

/* Upload a whole FP8 weight (host W [rows, cols] e4m3, host BF16 scales). */
int q35cu_weight_upload_fp8(const uint8_t *W, const uint16_t *scale_bf16,
                            uint32_t rows, uint32_t cols, q35cu_weight **out);
/* Upload the window [row0, row0+nrows) x [col0, col0+ncols) of a host FP8
 * weight [rows, cols] (a tensor-parallel shard).  row0 and col0 must be
 * multiples of 128 so no scale block is split. */
int q35cu_weight_upload_fp8_window(const uint8_t *W, const uint16_t *scale_bf16,
                                   uint32_t rows, uint32_t cols,
                                   uint32_t row0, uint32_t nrows,
                                   uint32_t col0, uint32_t ncols, q35cu_weight **out);
/* Upload a BF16 weight (the lm_head of q35_mm_bf16). */
int q35cu_weight_upload_bf16(const uint16_t *W, uint32_t rows, uint32_t cols,
                             q35cu_weight **out);
/* Generate a seeded synthetic FP8 weight directly in HBM: the window
 * [row0, +nrows) x [col0, +ncols) of a global [grows, gcols] matrix
 * W0 ~ N(0, stddev^2) quantised per global 128x128 block
 * (s = bf16(amax/448), W = e4m3_rne(W0/s)).  Every rank of a
 * tensor-parallel group generating its own window reproduces the shards of
 * one global matrix. */
int q35cu_weight_synth_fp8(uint64_t seed, float stddev, uint32_t grows, uint32_t gcols,
                           uint32_t row0, uint32_t nrows, uint32_t col0, uint32_t ncols,
                           q35cu_weight **out);
/* Copy a device weight back (W [rows, cols], BF16 scales) -- for checks. */
int q35cu_weight_download_fp8(const q35cu_weight *w, uint8_t *W, uint16_t *scale_bf16);
/* Make q35_mm_fp8 / _multi4 / _batch serve the host key (host_W, host_sc,
 * rows, cols) from the device weight w without an upload (a loader that
 * streamed the tensor to HBM itself).  w must outlive the binding. */
int q35cu_weight_bind(const uint8_t *host_W, const uint16_t *host_sc, const q35cu_weight *w);

/* Upload the matmul operands of one mapped safetensors shard now (base, len:
 * the whole file as mapped) and key them by their addresses in the mapping,
 * exactly as the first q35_mm_fp8 / q35_mm_bf16 call on them would: every
 * FP8 "X.weight" [rows, cols] with its BF16 "X.weight_scale_inv" grid (the
 * pair may span shards: the half seen first waits, by name, for the other),
 * and a BF16 "lm_head.weight".  The engine binds these pointers straight into
 * its mappings (qwen35-c/src/q35_model.c:252-273), so its first forward pass
 * then uploads nothing.  libq35plat's q35_plat_mmap_prefetch calls this when
 * libq35cuda is loaded (set Q35_PRELOAD=0 to keep first-touch uploads).
 * q35cu_preload_forget drops the unmatched halves that point into a mapping
 * about to be unmapped; q35cu_preload_bytes counts the bytes preloaded. */
int q35cu_preload_safetensors(const void *base, size_t len);
void q35cu_preload_forget(const void *base, size_t len);
size_t q35cu_preload_bytes(void);
void q35cu_weight_free(q35cu_weight *w);
uint32_t q35cu_weight_rows(const q35cu_weight *w);
uint32_t q35cu_weight_cols(const q35cu_weight *w);
size_t q35cu_weight_device_bytes(const q35cu_weight *w);

/* ---- device-pointer compute (asynchronous on `stream`) ----------------- */
/* Y[t, r] = sum_k X[t, k] * W[r, k] * s[r/128, k/128] for t < m, on the
 * CUDA cores in fp32 (the decode GEMV; q35_mm_fp8 / q35_mm_fp8_batch with
 * small n).  Deterministic; row results do not depend on m. */
int q35cu_gemv_fp8(const q35cu_weight *w, const float *X, uint32_t ldx, uint32_t m,
                   float *Y, uint32_t ldy, void *stream);
/* o[i] = silu(g[i]) * u[i] for i < n -- the engine's swiglu between the
 * gate/up and down projections (qwen35-c/src/q35_kern.c), used by the
 * decode-step harness to chain the projections. */
int q35cu_swiglu(const float *g, const float *u, float *o, size_t n, void *stream);
/* Up to four weights sharing X and cols in one launch (q35_mm_fp8_multi4);
 * w[s] == NULL skips segment s; Y[s] is [m, rows_s] (row stride rows_s). */
int q35cu_multi_fp8(const q35cu_weight *const w[4], const float *X, uint32_t ldx, uint32_t m,
                    float *const Y[4], void *stream);
/* Tensor-core GEMM for prefill: Y [m, rows] fp32 = Xb [m, cols] bf16 times
 * the dequantised weight, fp32 accumulation with per-128-K block-scale
 * promotion.  Needs cols % 16 == 0.  The caller provides a device workspace
 * of at least q35cu_gemm_fp8_workspace_bytes(m, cols) bytes (16-byte
 * aligned) for the prepared activations: two e4m3 terms per value with a
 * per-token power of two (exact down to 2^-13 of a row's largest magnitude,
 * within 2^-21 of it below; with Q35CU_GEMM_F16 set, f16 values, exact);
 * calls on different streams need different workspaces.  The library
 * allocates nothing here. */
size_t q35cu_gemm_fp8_workspace_bytes(uint32_t m, uint32_t cols);
int q35cu_gemm_fp8(const q35cu_weight *w, const uint16_t *Xb, uint32_t m,
                   float *Y, void *workspace, size_t workspace_bytes, void *stream);
/* q35cu_gemm_fp8 on fp32 activations X [m, cols] (device memory), rounded
 * to bf16 (nearest even) as they are prepared: the same results as
 * converting X to bf16 first and calling q35cu_gemm_fp8, without that
 * separate pass over X.  Same workspace. */
int q35cu_gemm_fp8_f32(const q35cu_weight *w, const float *X, uint32_t m,
                       float *Y, void *workspace, size_t workspace_bytes, void *stream);
/* Up to four prefill GEMMs on the same activations, as one: weight i (all
 * nw of them with the same cols) times X into Y[i] [m, rows_i], with one
 * preparation of X and one persistent launch over the weights' row blocks
 * together -- the projections that read one input (q | k | v, gate | up,
 * qkv | z) fill the GPU where a small one alone would not.  X [m, cols] is
 * bf16 bits (x_f32 = 0) or fp32 (x_f32 = 1, rounded to bf16).  Results are
 * those of q35cu_gemm_fp8 / q35cu_gemm_fp8_f32 weight by weight, bit for
 * bit.  nw in 1..4; same workspace as q35cu_gemm_fp8 (m, cols). */
int q35cu_gemm_fp8_multi(const q35cu_weight *const *w, uint32_t nw, const void *X, int x_f32,
                         uint32_t m, float *const *Y, void *workspace, size_t workspace_bytes,
                         void *stream);
/* The prefill GEMM of q35cu_gemm_fp8 on fp32 activations, for callers that
 * may not have the library allocate device memory and hold no workspace: a
 * serving process that reserved its HBM budget up front, or a loop that
 * cannot absorb the device synchronisation a cudaMalloc / cudaFree can
 * bring.  No counterpart in the reference (its matmuls run on host memory).
 *   X [m, cols] fp32 and Y [m, rows] fp32 are device memory owned by the
 *   caller; X is rounded to bf16 (the prefill contract) and prepared into
 *   fixed arrays compiled into the library (16 MiB of activations, 2 MiB of
 *   per-token scales) -- every GPU that loads the library holds them until
 *   exit -- so m * cols may be at most Q35CU_NOALLOC_MAX_ACTS; larger calls
 *   fail with Q35CU_ERR_ARG.
 *   All calls share those arrays: calls that overlap on the GPU race.
 *   The first call on a device looks up the array's address and configures
 *   the kernel; make it before any stream capture.  stream NULL = the
 *   legacy default stream.  Allocates nothing. */
#define Q35CU_NOALLOC_MAX_ACTS (8u << 20)
int q35cu_gemm_fp8_f32_noalloc(const q35cu_weight *w, const float *X, uint32_t m,
                               float *Y, void *stream);
/* Multi-token decode on the tensor cores with exact fp32 activations: Y [m,
 * rows] = X [m, cols] fp32 times the dequantised weight.  Each token row is
 * scaled by a power of two and, up to 48 tokens, split into five e4m3 terms
 * (to 2^-33 of the row's largest magnitude) multiplied on e4m3 tensor-core
 * MMAs; above 48 tokens (or with Q35CU_GEMV_TC_F16) into two f16 rows (hi =
 * f16(x), lo = f16(x - hi): about 22 bits of x).  The term columns are
 * summed in the epilogue; the weight streams once per token tile instead of
 * once per 4 tokens.  Meets the decode GEMV's per-element bound (guarded
 * 1e-5) but is not bit-identical to q35cu_gemv_fp8.  q35_mm_fp8_batch uses
 * it for batches of 16 (Q35CU_GEMV_TC_MIN_TOKENS) to 127 tokens.  cols % 16
 * == 0; workspace >= q35cu_gemv_fp8_tc_workspace_bytes(m, cols), 16-byte
 * aligned. */
size_t q35cu_gemv_fp8_tc_workspace_bytes(uint32_t m, uint32_t cols);
int q35cu_gemv_fp8_tc(const q35cu_weight *w, const float *X, uint32_t m, float *Y, void *workspace,
                      size_t workspace_bytes, void *stream);
/* The tensor-core GEMM is persistent (one CTA per SM).  When a caller runs
 * other work beside it -- a collective on another stream overlapping the
 * next token slab's GEMM -- a CTA that finds its SM busy starts late and
 * holds up its share of the tiles.  q35cu_gemm_reserve_sms(n) makes later
 * GEMM launches of this process use n SMs fewer (0 = all; the default). */
int q35cu_gemm_reserve_sms(int n);
/* fp32 -> bf16 (nearest even) conversion of n values. */
int q35cu_f32_to_bf16(const float *x, uint16_t *y, size_t n, void *stream);
/* y[rows] = W x for a bf16 weight (q35_mm_bf16). */
int q35cu_gemv_bf16(const q35cu_weight *w, const float *x, float *y, void *stream);

/* ---- tensor parallel (NCCL over NVLink) -------------------------------- */
/* The reference is single-process; these are new.  Column-parallel layers
 * (gate/up/qkv/z/q/k/v) split W by rows and all-gather Y; row-parallel
 * layers (down/o/out) split W by columns and all-reduce Y. */
typedef enum { Q35CU_SHARD_COLUMN = 0, Q35CU_SHARD_ROW = 1 } q35cu_shard_mode;
/* Host-only: the window of W [rows, cols] held by `rank` of `world`
 * (128-aligned; the last rank takes the remainder).  No GPU needed. */
int q35cu_shard_window(uint32_t rows, uint32_t cols, int mode, int rank, int world,
                       uint32_t *row0, uint32_t *nrows, uint32_t *col0, uint32_t *ncols);
int q35cu_nccl_unique_id(void *out, size_t cap);   /* cap >= 128 */
int q35cu_tp_init(int rank, int world, const void *id, size_t idlen);
int q35cu_tp_world(void);
int q35cu_tp_rank(void);
int q35cu_tp_finalize(void);
int q35cu_allreduce_f32(float *buf, size_t n, void *stream);
int q35cu_allgather_f32(const float *send, float *recv, size_t n_per_rank, void *stream);
/* One-shot collectives over NVLink peer memory for the small vectors a
 * tensor-parallel decode step exchanges (no NCCL call; the reference has no
 * counterpart).  Every rank owns an exchange area in its HBM:
 *   1. q35cu_p2p_handle(h, cap): allocates this rank's area (on the current
 *      device) and writes its CUDA IPC handle (Q35CU_P2P_HANDLE_BYTES bytes);
 *   2. the caller gathers every rank's handle (rank order, any transport);
 *   3. q35cu_p2p_open(rank, world, handles, Q35CU_P2P_HANDLE_BYTES) maps the
 *      peers' areas (world <= 8, one process per GPU).
 * The collectives are then asynchronous on `stream` and may be captured in a
 * CUDA graph; every rank must issue the same sequence of them.  The sum is
 * taken in rank order, so all ranks get the same bits, run after run.  At
 * most q35cu_p2p_max_elems() values per rank per call (larger exchanges stay
 * on NCCL).  in == out is allowed.  q35cu_p2p_close() unmaps and frees (call
 * it on every rank once no collective is in flight). */
#define Q35CU_P2P_HANDLE_BYTES 64
int q35cu_p2p_handle(void *out, size_t cap);
int q35cu_p2p_open(int rank, int world, const void *handles, size_t handle_bytes);
int q35cu_p2p_close(void);
size_t q35cu_p2p_max_elems(void);
int q35cu_p2p_allreduce_f32(const float *in, float *out, size_t n, void *stream);
int q35cu_p2p_allgather_f32(const float *send, float *recv, size_t n_per_rank, void *stream);
/* The decode GEMV (one token) with the tensor-parallel exchange fused into
 * its epilogue over the same peer memory (q35cu_p2p_open first): every rank
 * splits the rows over CTAs the same way, so each CTA publishes its output
 * rows to every rank and waits only for its peers' copies of those rows --
 * no separate collective kernel.
 *   Q35CU_TP_ALLREDUCE (row-parallel: down/o/out): Y[s] = the sum over ranks
 *     (in rank order) of every rank's product;
 *   Q35CU_TP_ALLGATHER (column-parallel: gate/up/qkv/z/q/k/v): Y[s] as
 *     q35cu_multi_fp8, and gathered[q * R + v] = rank q's row v, with v the
 *     call's row index over its segments in order and R their total rows
 *     (the layout of q35cu_allgather_f32 on the packed outputs).
 * X is [cols] fp32.  Every rank must make the same sequence of calls. */
typedef enum { Q35CU_TP_ALLREDUCE = 1, Q35CU_TP_ALLGATHER = 2 } q35cu_tp_mode;
int q35cu_multi_fp8_tp(const q35cu_weight *const w[4], const float *X, float *const Y[4], int mode,
                       float *gathered, void *stream);
int q35cu_gemv_fp8_tp(const q35cu_weight *w, const float *X, float *Y, int mode, float *gathered, void *stream);

/* A decode chain: a fixed sequence of one-token decode GEMVs (each up to four
 * weights sharing X, optionally with the fused tensor-parallel exchange
 * above) run by one cooperative kernel launch.  The CTAs stay resident across
 * the ops and wait on a grid barrier before each op after the first -- with
 * that op's first weights already in flight -- so no launch ramp or tail
 * separates two projections.  Ops run in the order added; op k may read what
 * ops < k wrote.  X and Y are device pointers fixed when the op is added
 * (their contents may change between runs).  The first run lays out and
 * uploads the op table (synchronously): make it before any stream capture;
 * later runs are a single asynchronous launch and may be captured.  The
 * reference has no counterpart: it calls q35_mm_fp8 / _multi4 per projection
 * from its layer code (qwen35-c/src/q35_model.c, q35_deltanet.c, q35_attn.c). */
typedef struct q35cu_chain q35cu_chain;
int q35cu_chain_create(q35cu_chain **out);
int q35cu_chain_add(q35cu_chain *c, const q35cu_weight *const w[4], const float *X, float *const Y[4], int mode,
                    float *gathered);
int q35cu_chain_run(q35cu_chain *c, void *stream);
void q35cu_chain_free(q35cu_chain *c);

/* ---- info --------------------------------------------------------------- */
const char *q35cu_build_info(void);
/* Kernel launches this library issued since load (all entry points). */
uint64_t q35cu_launch_count(void);
/* The device status word of the current device: 0, or the q35cu_status of
 * a bounded device-side wait that gave up (Q35CU_ERR_TIMEOUT) since the
 * last clear.  Asynchronous device-pointer callers check it after a
 * synchronisation; the q35_mm_* entry points check it on every call. */
int q35cu_device_status(uint32_t *status, int clear);
/* Where the tensor-core GEMM wait that last gave up was: out[0] = role
 * (1 activation producer, 2 weight producer, 3 MMA issuer, 4 converter,
 * 5 epilogue, 6 wind-down), out[1] = CTA, out[2] = 128-column block index
 * within the CTA's walk, out[3] = thread.  Meaningful after
 * q35cu_device_status reported Q35CU_ERR_TIMEOUT from a GEMM (the q35_mm_*
 * entry points put it in their error message). */
int q35cu_gemm_timeout_info(uint32_t out[4]);

#ifdef __cplusplus
}
#endif
#endif /* Q35CU_H */
