// Internal declarations shared by the libq35cuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "q35cu.h"

#define Q35CU_STR2(x) #x
#define Q35CU_STR(x) Q35CU_STR2(x)

struct q35cu_weight {
    int kind;            // 0 = FP8 e4m3 + fp32 block scales, 1 = BF16
    uint32_t rows, cols; // logical shape of the device tensor
    void *d_w;           // [rows, cols] bytes (fp8) or bf16
    float *d_s;          // [rows_blk, cols_blk] fp32 scales (fp8 only)
    uint32_t rows_blk, cols_blk;
    size_t bytes;        // device bytes held
    int device;
    uint32_t has_nan;    // FP8 weight holds NaN codes 0x7F / 0xFF (set by the upload scan)
};

namespace q35cu {

// ---- error plumbing (shim.cu) ----
int set_error(int code, const char *fmt, ...);
int cuda_error(cudaError_t e, const char *what);
#define Q35CU_CUDA(call)                                         \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return q35cu::cuda_error(e_, #call); \
    } while (0)

int device_sms();
void count_launch(uint64_t n = 1);
cudaStream_t default_stream();

// ---- device memory with the budget check (shim.cu) ----
int dev_alloc(void **p, size_t bytes);
void dev_free(void *p, size_t bytes);

// ---- kernels (gemv.cu / gemm.cu / synth.cu) ----
struct GemvSeg {
    const uint8_t *W;   // [rows, K] (fp8 bytes, or bf16 when kind == 1)
    const float *S;     // [ceil(rows/128), ceil(K/128)] (fp8 only)
    float *Y;           // output for this segment, token-major [m, ldy]
    uint32_t rows;
    uint32_t ldy;
    uint32_t has_nan;   // weight holds e4m3 NaN codes
};

// tensor-parallel epilogue of the decode GEMV (m = 1): 0 none, 1 all-reduce
// the outputs across ranks (Y = sum of every rank's product), 2 all-gather
// them (Y as usual, plus gathered[q * R + v] = rank q's virtual row v)
struct GemvTp {
    int mode = 0;
    float *gathered = nullptr;
};
// Completion signal of a host-pointer call: the launch's last CTA to finish
// writes {seq, the device status word} into flag (host-mapped memory), after
// every CTA's outputs are visible system-wide; count (device memory, zero
// between launches) counts the CTAs out.  Only the tensor-core decode GEMV
// (FP8, cols % 128 == 0, 16-byte aligned) signals: launch_gemv refuses a
// signal for any other kernel.
struct HostSignal {
    uint32_t *count = nullptr;
    uint32_t *flag = nullptr;
    uint32_t seq = 0;
};
int launch_gemv(int kind, const GemvSeg *segs, int nseg, const float *X,
                uint32_t K, uint32_t ldx, uint32_t m, cudaStream_t st, const GemvTp &tp = GemvTp{},
                const HostSignal *sig = nullptr);
// the decode chain: op descriptors are opaque bytes (chain_op_bytes each)
size_t chain_op_bytes();
int chain_build_op(const GemvSeg *segs, int nseg, const float *X, uint32_t K, const GemvTp &tp, void *out);
int chain_layout(void *ops, uint32_t nops, uint32_t layout_out[5]);
int launch_chain(const void *d_ops, uint32_t nops, uint32_t *d_bar, const uint32_t layout[5], cudaStream_t st);
int launch_swiglu(const float *g, const float *u, float *o, size_t n, cudaStream_t st);
void gemv_geometry(int kind, uint32_t K, uint32_t *threads, uint32_t *passes);
int device_status(uint32_t *status, bool clear);
int scan_nan_codes(const uint8_t *W, size_t bytes, uint32_t *d_flag, cudaStream_t st, bool *has_nan);

// prefill GEMM: activations prepared once per call (f16, per-token power-of-two
// scale) into a workspace of gemm_workspace_bytes(m, K): Xh [m, K] f16 at
// offset 0, tscale [m] fp32 after it (256-byte aligned)
size_t gemm_workspace_bytes(uint32_t m, uint32_t K);
int launch_gemm_prep(const void *X, bool f32, uint32_t m, uint32_t K, uint16_t *Xh, float *tscale,
                     cudaStream_t st);
int launch_gemm_fp8(const q35cu_weight *w, const uint16_t *Xh, const float *tscale, uint32_t m, float *Y,
                    cudaStream_t st, bool pair = false);
// the prefill GEMM on bf16-valued activations (X bf16 bits, or fp32 rounded
// to bf16 when f32): activation preparation into workspace (at least
// gemm_workspace_bytes(m, K) bytes, 16-byte aligned) + the tensor-core GEMM
// (fp8 operands by default; Q35CU_GEMM_F16 selects the f16-operand kernel)
int launch_gemm_bf16(const q35cu_weight *w, const void *X, bool f32, uint32_t m, float *Y, void *workspace,
                     cudaStream_t st);
// the same over nw (1..4) weights of equal cols that multiply the same X:
// one preparation and one launch, weight i into Y[i] [m, rows_i]
int launch_gemm_bf16_multi(const q35cu_weight *const *w, float *const *Y, uint32_t nw, const void *X, bool f32,
                           uint32_t m, void *workspace, cudaStream_t st);
// multi-token decode on the tensor cores, fp32 activations split hi/lo
size_t gemm_exact_workspace_bytes(uint32_t m, uint32_t K);
int launch_gemm_exact(const q35cu_weight *w, const float *X, uint32_t m, float *Y, void *workspace,
                      cudaStream_t st);
int launch_f32_to_bf16(const float *x, uint16_t *y, size_t n, cudaStream_t st);
int gemm_status(uint32_t *status, bool clear);
int gemm_reserve_sms(int n);
// role, CTA, block and thread of the GEMM wait that last gave up
int gemm_timeout_info(uint32_t out[4]);
// device addresses of the three status words (GEMV and generic kernels,
// GEMM, peer-memory collectives) on the current device, for a host call that
// reads them together with its output in one copy
uint32_t *device_status_word();
uint32_t *gemm_status_word();
uint32_t *p2p_status_word();
int p2p_status(uint32_t *status, bool clear);
struct P2PView;
// the mapped exchange areas of q35cu_p2p_open (false if not open)
bool p2p_view(P2PView *out);
int launch_bf16_to_f32_scales(const uint16_t *src, float *dst, size_t n, cudaStream_t st);
int launch_f32_to_bf16_scales(const float *src, uint16_t *dst, size_t n, cudaStream_t st);
int launch_synth_fp8(uint64_t seed, float stddev, uint32_t grows, uint32_t gcols,
                     uint32_t row0, uint32_t col0, uint32_t nrows, uint32_t ncols,
                     uint8_t *W, float *S, cudaStream_t st);
int launch_fill_nan(float *p, size_t n, cudaStream_t st);

}  // namespace q35cu
