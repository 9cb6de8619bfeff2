/*
 * q35_mm.h -- drop-in boundary: the FP8/BF16 matmul entry points of the
 * qwen35-c engine, served by libq35cuda.so on an sm_100a GPU.
 *
 * Every declaration below keeps the exact C signature of
 * qwen35-c/include/q35/q35_mm.h (lines cited per entry), so the engine's
 * callers (q35_model.c, q35_deltanet.c, q35_attn.c) link unchanged against
 * libq35cuda.so in place of q35_mm.c.
 *
 * Shared contract (same as the reference):
 *   - all pointers are caller-owned HOST memory; W and the scale grid are
 *     treated as immutable for the life of the process (they point into
 *     read-only safetensors mappings), x / y are scratch reused across calls;
 *   - W is row-major [rows, cols] e4m3fn bytes, the scale grid is BF16
 *     [ceil(rows/128), ceil(cols/128)], one value per 128x128 block;
 *   - the calls return void and are synchronous: y is complete on return.
 *
 * What changes behind the signatures (see q35cu.h for the knobs):
 *   - the first call that sees a (W, scale, rows, cols) uploads the weight
 *     to HBM once (scales widened to fp32, exact); later calls reuse it;
 *   - q35_mm_fp8_batch with n >= 128 tokens (and cols % 16 == 0) runs the
 *     tensor-core path, which rounds X to bf16 (relative L2 error of Y
 *     <= 5e-3); smaller n keeps fp32 activations on the CUDA cores;
 *   - a CUDA failure aborts with a message by default (the signatures have
 *     no error channel); q35cu_set_error_mode() switches to record-and-return.
 */
#ifndef Q35_MM_H
#define Q35_MM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* e4m3fn byte -> f32 table (256 entries), filled by q35_mm_init().
 * Replaces qwen35-c/include/q35/q35_mm.h:16 (also read by q35_model.c:49). */
extern float q35_mm_fp8_lut[256];

/* Build the table; idempotent. Replaces qwen35-c/include/q35/q35_mm.h:17. */
void q35_mm_init(void);

/* e4m3fn decode: bias 7, subnormal step 2^-9, 0x7F/0xFF -> NaN, no inf.
 * Replaces qwen35-c/include/q35/q35_mm.h:19. */
float q35_mm_e4m3_to_f32(uint8_t v);

/* bf16 storage bits -> f32, exact. Replaces qwen35-c/include/q35/q35_mm.h:22. */
float q35_mm_bf16_to_f32(uint16_t v);

/* y[rows] = (W (.) scale) x.  Replaces qwen35-c/include/q35/q35_mm.h:24-26. */
void q35_mm_fp8(const uint8_t *W, const uint16_t *scale_bf16,
                uint32_t rows, uint32_t cols,
                const float *x, float *y);

/* Y = X (W (.) scale)^T with X [n, cols] and Y TOKEN-MAJOR [n, rows]
 * (Y[t * rows + r], as qwen35-c/src/q35_mm.c:168 writes it).
 * Replaces qwen35-c/include/q35/q35_mm.h:32-34. */
void q35_mm_fp8_batch(const uint8_t *W, const uint16_t *scale_bf16,
                      uint32_t rows, uint32_t cols, uint32_t n,
                      const float *X, float *Y);

/* Up to four matvecs sharing x and cols in one launch; rows[s] == 0 skips
 * segment s.  Replaces qwen35-c/include/q35/q35_mm.h:40-42. */
void q35_mm_fp8_multi4(const uint8_t *W[4], const uint16_t *sc[4],
                       uint32_t rows[4], uint32_t cols,
                       const float *x, float *y[4]);

/* y[rows] = W x with W bf16 [rows, cols] (the lm_head).
 * Replaces qwen35-c/include/q35/q35_mm.h:44-45. */
void q35_mm_bf16(const uint16_t *W, uint32_t rows, uint32_t cols,
                 const float *x, float *y);

/* Which implementation ran: "sm_100a".  Replaces qwen35-c/include/q35/q35_mm.h:48. */
const char *q35_mm_impl_fp8(void);

#ifdef __cplusplus
}
#endif
#endif /* Q35_MM_H */
