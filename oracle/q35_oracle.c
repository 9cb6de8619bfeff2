/*
 * q35_oracle.c -- CPU ORACLE for the FP8 block-scaled matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline / reference arm load it, and only as the checker.
 *
 * It restates, in plain scalar C, the arithmetic of qwen35-c's FP8 matmul:
 *
 *   - e4m3fn decode (bias 7, subnormal step 2^-9, 0x7F/0xFF -> NaN, no inf):
 *     qwen35-c/src/q35_mm.c:22-37
 *   - bf16 bits -> f32 (<<16, exact): qwen35-c/src/q35_mm.c:46-52
 *   - one output row (mm_fp8_row, scalar branch): eight lanes indexed by
 *     k & 7, each updated by fmaf((lut[w_k] * s_blk), x_k, lane), the block
 *     scale re-read every 128 columns, then the lanes folded left to right:
 *     qwen35-c/src/q35_mm.c:88-142 (the AVX2 branch is bit-identical to it)
 *   - q35_mm_fp8 (matvec):            qwen35-c/src/q35_mm.c:144-153
 *   - q35_mm_fp8_batch (Y token-major [n, rows]): qwen35-c/src/q35_mm.c:158-172
 *   - q35_mm_fp8_multi4:              qwen35-c/src/q35_mm.c:176-198
 *   - q35_mm_bf16 (matvec, 8 lanes):  qwen35-c/src/q35_mm.c:211-246
 *   - block quantizer (amax/448, scale rounded to bf16, nearest-even e4m3):
 *     qwen35-c/src/q35_model.c:30-57 and :327-343
 *
 * Because every step (lane assignment, operation order, FMA vs. multiply)
 * follows the reference, this file reproduces the reference outputs
 * bit-for-bit; tests check that against the reference's own FNV-1a anchors
 * and, when the reference sources are present, against oracle/_ref.
 *
 * It also holds what the checks need beyond the reference: an fp64
 * reference product and the seeded synthetic weight generator used by the
 * benchmark configurations (same counter-based RNG as the device generator).
 *
 * Build: oracle/Makefile (-O2 -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* scalar decoders                                                     */
/* ------------------------------------------------------------------ */

ORC_API float orc_e4m3_to_f32(uint8_t b)
{
    int neg = b >> 7;
    int e = (b >> 3) & 15;
    int m = b & 7;
    float mag;
    if (e == 15 && m == 7) return NAN;          /* 0x7F / 0xFF */
    if (e == 0) mag = (float)m / 512.0f;        /* m * 2^-9 */
    else mag = ldexpf((float)(8 + m), e - 10);  /* (1 + m/8) * 2^(e-7) */
    return neg ? -mag : mag;
}

ORC_API float orc_bf16_to_f32(uint16_t h)
{
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

ORC_API uint16_t orc_f32_to_bf16_rne(float f)
{
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
        return (uint16_t)((u >> 16) | 0x40u);   /* quiet NaN */
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* nearest e4m3fn, ties to even mantissa, saturating to +-448 */
ORC_API uint8_t orc_f32_to_e4m3_rne(float v)
{
    uint8_t sign = signbit(v) ? 0x80u : 0u;
    float a = fabsf(v);
    if (a != a) return 0x7Fu;
    if (a >= 448.0f) return sign | 0x7Eu;
    if (a < 0.015625f) {                       /* below 2^-6: step 2^-9 */
        float q = rintf(a * 512.0f);            /* 0..8, 8 == 2^-6 */
        return sign | (uint8_t)q;
    }
    int e;
    frexpf(a, &e);                              /* a = f * 2^e, f in [0.5,1) */
    e -= 1;                                     /* a in [2^e, 2^(e+1)) */
    float q = rintf(ldexpf(a, 3 - e));          /* 8..16 */
    int qi = (int)q;
    if (qi == 16) { qi = 8; e += 1; }
    if (e > 8 || (e == 8 && qi > 14)) return sign | 0x7Eu;
    return sign | (uint8_t)(((e + 7) << 3) | (qi - 8));
}

static float g_lut[256];
static int g_lut_ready;

static void lut_init(void)
{
    if (g_lut_ready) return;
    for (int i = 0; i < 256; i++) g_lut[i] = orc_e4m3_to_f32((uint8_t)i);
    g_lut_ready = 1;
}

ORC_API const float *orc_lut(void)
{
    lut_init();
    return g_lut;
}

/* ------------------------------------------------------------------ */
/* the reference's row dot product                                     */
/* ------------------------------------------------------------------ */

static float row_dot_fp8(const uint8_t *wr, const uint16_t *sc_row,
                         uint32_t cols, const float *x)
{
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (uint32_t k0 = 0; k0 < cols; k0 += 128) {
        uint32_t k1 = k0 + 128 < cols ? k0 + 128 : cols;
        float s = orc_bf16_to_f32(sc_row[k0 / 128]);
        for (uint32_t k = k0; k < k1; k++) {
            float ws = g_lut[wr[k]] * s;            /* exact: 4 x 8 bits */
            lane[k & 7] = fmaf(ws, x[k], lane[k & 7]);
        }
    }
    float sum = 0.0f;
    for (int j = 0; j < 8; j++) sum += lane[j];
    return sum;
}

ORC_API void orc_mm_fp8(const uint8_t *W, const uint16_t *sc, uint32_t rows,
                        uint32_t cols, const float *x, float *y)
{
    lut_init();
    uint32_t scc = (cols + 127) / 128;
    #pragma omp parallel for schedule(static)
    for (uint32_t r = 0; r < rows; r++)
        y[r] = row_dot_fp8(W + (size_t)r * cols, sc + (size_t)(r / 128) * scc, cols, x);
}

ORC_API void orc_mm_fp8_batch(const uint8_t *W, const uint16_t *sc, uint32_t rows,
                              uint32_t cols, uint32_t n, const float *X, float *Y)
{
    lut_init();
    uint32_t scc = (cols + 127) / 128;
    #pragma omp parallel for schedule(static)
    for (uint32_t r = 0; r < rows; r++)
        for (uint32_t t = 0; t < n; t++)
            Y[(size_t)t * rows + r] = row_dot_fp8(W + (size_t)r * cols,
                                                  sc + (size_t)(r / 128) * scc, cols,
                                                  X + (size_t)t * cols);
}

ORC_API void orc_mm_fp8_multi4(const uint8_t *const W[4], const uint16_t *const sc[4],
                               const uint32_t rows[4], uint32_t cols,
                               const float *x, float *const y[4])
{
    for (int s = 0; s < 4; s++)
        if (rows[s]) orc_mm_fp8(W[s], sc[s], rows[s], cols, x, y[s]);
}

ORC_API void orc_mm_bf16(const uint16_t *W, uint32_t rows, uint32_t cols,
                         const float *x, float *y)
{
    #pragma omp parallel for schedule(static)
    for (uint32_t r = 0; r < rows; r++) {
        const uint16_t *wr = W + (size_t)r * cols;
        float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (uint32_t k = 0; k < cols; k++)
            lane[k & 7] = fmaf(orc_bf16_to_f32(wr[k]), x[k], lane[k & 7]);
        float sum = 0.0f;
        for (int j = 0; j < 8; j++) sum += lane[j];
        y[r] = sum;
    }
}

/* ------------------------------------------------------------------ */
/* fp64 reference and error floor                                      */
/* ------------------------------------------------------------------ */

/* Y64[t, r] = sum_k (e4m3(W[r,k]) * s[r/128, k/128]) * X[t, k] in double;
 * ABS[t, r] = sum_k |...| (the conditioning of each output). */
ORC_API void orc_mm_fp8_f64(const uint8_t *W, const uint16_t *sc, uint32_t rows,
                            uint32_t cols, uint32_t n, const float *X,
                            double *Y64, double *ABS)
{
    lut_init();
    uint32_t scc = (cols + 127) / 128;
    #pragma omp parallel for schedule(static)
    for (uint32_t r = 0; r < rows; r++) {
        const uint8_t *wr = W + (size_t)r * cols;
        const uint16_t *sr = sc + (size_t)(r / 128) * scc;
        for (uint32_t t = 0; t < n; t++) {
            const float *xt = X + (size_t)t * cols;
            double acc = 0.0, mag = 0.0;
            for (uint32_t k = 0; k < cols; k++) {
                double p = (double)g_lut[wr[k]] * (double)orc_bf16_to_f32(sr[k / 128]) * (double)xt[k];
                acc += p;
                mag += fabs(p);
            }
            Y64[(size_t)t * rows + r] = acc;
            if (ABS) ABS[(size_t)t * rows + r] = mag;
        }
    }
}

ORC_API uint64_t orc_fnv1a(const void *p, size_t n)
{
    const uint8_t *c = (const uint8_t *)p;
    uint64_t h = 1469598103934665603ULL;
    for (size_t i = 0; i < n; i++) { h ^= c[i]; h *= 1099511628211ULL; }
    return h;
}

/* ------------------------------------------------------------------ */
/* seeded synthetic weights (same algorithm as the device generator)   */
/* ------------------------------------------------------------------ */

/* splitmix64 finaliser (Steele, Lea, Flood 2014) */
static inline uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* standard normal for global element g of stream `seed` (Box-Muller on
 * two 24-bit uniforms drawn from one 64-bit hash) */
ORC_API float orc_synth_normal(uint64_t seed, uint64_t g)
{
    uint64_t h = mix64(seed * 0x9E3779B97F4A7C15ULL + (g + 1) * 0xD1B54A32D192ED03ULL);
    float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777216.0f);   /* (0,1] */
    float u2 = (float)(uint32_t)((h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f); /* [0,1) */
    return sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
}

/* Block-quantised FP8 weight, a [nrows x ncols] window at (row0, col0) of
 * a global [grows x gcols] matrix W0 ~ N(0, std^2):
 *   s   = bf16_rne(amax(block) / 448)   per global 128x128 block
 *   W   = e4m3_rne(clamp(W0 / s, +-448)), all-zero block -> s = 0, W = 0
 * row0/col0 must be multiples of 128 (shards never split a block).
 * W: [nrows, ncols] bytes, SC: [ceil(nrows/128), ceil(ncols/128)] bf16. */
ORC_API int orc_synth_fp8(uint64_t seed, float stddev, uint32_t grows, uint32_t gcols,
                          uint32_t row0, uint32_t col0, uint32_t nrows, uint32_t ncols,
                          uint8_t *W, uint16_t *SC)
{
    if ((row0 & 127) || (col0 & 127)) return -1;
    if (row0 + nrows > grows || col0 + ncols > gcols) return -2;
    uint32_t br = (nrows + 127) / 128, bc = (ncols + 127) / 128;
    #pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (uint32_t bi = 0; bi < br; bi++) {
        for (uint32_t bj = 0; bj < bc; bj++) {
            uint32_t r0 = bi * 128, c0 = bj * 128;
            /* the whole global block decides amax, even if the window
               only holds part of it (it never does: windows are aligned) */
            uint32_t gr0 = row0 + r0, gc0 = col0 + c0;
            uint32_t gr1 = gr0 + 128 < grows ? gr0 + 128 : grows;
            uint32_t gc1 = gc0 + 128 < gcols ? gc0 + 128 : gcols;
            float amax = 0.0f;
            for (uint32_t r = gr0; r < gr1; r++)
                for (uint32_t c = gc0; c < gc1; c++) {
                    float v = fabsf(stddev * orc_synth_normal(seed, (uint64_t)r * gcols + c));
                    if (v > amax) amax = v;
                }
            float s = orc_bf16_to_f32(orc_f32_to_bf16_rne(amax / 448.0f));
            SC[(size_t)bi * bc + bj] = orc_f32_to_bf16_rne(s);
            for (uint32_t r = gr0; r < gr1; r++) {
                uint32_t lr = r - row0;
                if (lr >= nrows) break;
                for (uint32_t c = gc0; c < gc1; c++) {
                    uint32_t lc = c - col0;
                    if (lc >= ncols) break;
                    float v = stddev * orc_synth_normal(seed, (uint64_t)r * gcols + c);
                    W[(size_t)lr * ncols + lc] = s == 0.0f ? 0 : orc_f32_to_e4m3_rne(v / s);
                }
            }
        }
    }
    return 0;
}

/* fp32 N(0,1) activations, optionally rounded to bf16 values */
ORC_API void orc_synth_act(uint64_t seed, size_t n, int round_bf16, float *out)
{
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
        float v = orc_synth_normal(seed, i);
        out[i] = round_bf16 ? orc_bf16_to_f32(orc_f32_to_bf16_rne(v)) : v;
    }
}

ORC_API int orc_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
