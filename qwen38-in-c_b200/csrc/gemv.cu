// Weight-streaming GEMV for the decode path (M <= 64 tokens), sm_100a.
//
// Replaces the CPU row loop of qwen35-c/src/q35_mm.c:88-198 (mm_fp8_row,
// q35_mm_fp8, q35_mm_fp8_batch, q35_mm_fp8_multi4) and the BF16 matvec
// q35_mm_bf16 (qwen35-c/src/q35_mm.c:211-246).
//
// Roofline: HBM.  Each weight byte is read from DRAM exactly once per token
// tile; the algorithmic traffic of one launch is rows*cols weight bytes
// (x2 for bf16) + 4*ceil(rows/128)*ceil(cols/128) scale bytes
// + 4*m*cols activation bytes + 4*m*rows output bytes.
//
// Work decomposition (one CTA = 8 warps):
//   task   = kRows (4) consecutive weight rows x the full K range;
//   wpt    = warps that split one task's K range (1, 2, 4 or 8), chosen per
//            weight from (rows, cols) only, so a row's arithmetic never
//            depends on m or on which other weights share the launch;
//   chunk  = 32 lanes x 16 bytes of one row (512 fp8 / 256 bf16 values);
//            warp `part` of a task takes chunks part, part+wpt, ...
// Each lane streams 16-byte vectors of kRows rows with L1-bypassing loads,
// keeps the next chunk's loads in flight while it converts and multiplies
// the current one, converts e4m3 pairs with the hardware cvt (exact; NaN
// bytes stay NaN), and applies the block scale once per 16-value group:
//   acc_r = fma(s[r/128, k/128], sum_{j<16} w_rj * x_j, acc_r).
// The lanes of a warp are folded with an xor butterfly, the warps of a task
// in fixed order through shared memory: no atomics, deterministic, and the
// batch/multi entry points give bit-identical rows to the single matvec,
// as the reference's test_batch_mm requires (qwen35-c/tests/test_batch_mm.c).
#include <cuda_fp16.h>

#include "q35cu_internal.h"

namespace q35cu {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 4;

struct Args {
    GemvSeg seg[4];
    const float *X;
    uint32_t K, ldx, m, kblocks;
    int nseg;
};

__device__ __forceinline__ uint4 ld_stream(const void *p)
{
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// four e4m3 bytes (little-endian in w) -> four exact floats
__device__ __forceinline__ void e4m3x4(uint32_t w, float *f)
{
    uint32_t h01, h23;
    asm("{\n\t.reg .b16 lo, hi;\n\t"
        "mov.b32 {lo, hi}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
        "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
        : "=r"(h01), "=r"(h23)
        : "r"(w));
    float2 a = __half22float2(*reinterpret_cast<__half2 *>(&h01));
    float2 b = __half22float2(*reinterpret_cast<__half2 *>(&h23));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

// two bf16 (little-endian in w) -> two exact floats
__device__ __forceinline__ void bf16x2(uint32_t w, float *f)
{
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xFFFF0000u);
}

template <int KIND>
struct Fmt {
    static constexpr uint32_t kPer = KIND == 0 ? 16 : 8;  // values per 16-byte vector
    static constexpr uint32_t kEsz = KIND == 0 ? 1 : 2;   // bytes per value
    __device__ static __forceinline__ void unpack(const uint4 &v, float *f)
    {
        if constexpr (KIND == 0) {
            e4m3x4(v.x, f); e4m3x4(v.y, f + 4); e4m3x4(v.z, f + 8); e4m3x4(v.w, f + 12);
        } else {
            bf16x2(v.x, f); bf16x2(v.y, f + 2); bf16x2(v.z, f + 4); bf16x2(v.w, f + 6);
        }
    }
};

template <int KIND, int MT>
__global__ void __launch_bounds__(kThreads) gemv_vec_kernel(const __grid_constant__ Args a)
{
    using F = Fmt<KIND>;
    constexpr uint32_t P = F::kPer;
    __shared__ float red[kWarps][kRows * MT];

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t cta = blockIdx.x;
    int s = 0;
    if (a.nseg > 1 && cta >= a.seg[1].cta_begin) s = 1;
    if (a.nseg > 2 && cta >= a.seg[2].cta_begin) s = 2;
    if (a.nseg > 3 && cta >= a.seg[3].cta_begin) s = 3;
    const GemvSeg g = a.seg[s];
    const uint32_t wpt = g.wpt;
    const uint32_t task = (cta - g.cta_begin) * (kWarps / wpt) + warp / wpt;
    const uint32_t part = warp % wpt;
    const uint32_t r0 = task * kRows;
    const uint32_t t0 = blockIdx.y * MT;
    const uint32_t K = a.K;

    float acc[kRows][MT];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = 0.f;

    if (r0 < g.rows) {
        const uint32_t nchunks = (K + 32 * P - 1) / (32 * P);
        const uint8_t *wrow = g.W + (size_t)r0 * K * F::kEsz;
        const float *srow = KIND == 0 ? g.S + (size_t)(r0 >> 7) * a.kblocks : nullptr;
        bool rv[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) rv[r] = r0 + r < g.rows;

        uint4 wc[kRows], wn[kRows];
        auto load = [&](uint4 *w, uint32_t c) {
            const uint32_t k = c * 32 * P + lane * P;
#pragma unroll
            for (int r = 0; r < kRows; ++r)
                w[r] = (k < K && rv[r]) ? ld_stream(wrow + ((size_t)r * K + k) * F::kEsz)
                                        : make_uint4(0, 0, 0, 0);
        };
        uint32_t c = part;
        if (c < nchunks) load(wc, c);
#pragma unroll 1
        for (; c < nchunks; c += wpt) {
            if (c + wpt < nchunks) load(wn, c + wpt);
            const uint32_t k = c * 32 * P + lane * P;
            if (k < K) {
                const float sc = KIND == 0 ? __ldg(srow + (k >> 7)) : 1.f;
                float wf[kRows][P];
#pragma unroll
                for (int r = 0; r < kRows; ++r) F::unpack(wc[r], wf[r]);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    if (t0 + t < a.m) {
                        float xv[P];
                        const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)(t0 + t) * a.ldx + k);
#pragma unroll
                        for (int q = 0; q < (int)P / 4; ++q) {
                            float4 v = __ldg(xp + q);
                            xv[4 * q] = v.x; xv[4 * q + 1] = v.y; xv[4 * q + 2] = v.z; xv[4 * q + 3] = v.w;
                        }
#pragma unroll
                        for (int r = 0; r < kRows; ++r) {
                            float d = 0.f;
#pragma unroll
                            for (int j = 0; j < (int)P; ++j) d = fmaf(wf[r][j], xv[j], d);
                            acc[r][t] = fmaf(sc, d, acc[r][t]);
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kRows; ++r) wc[r] = wn[r];
        }
    }

    // fold the 32 lanes (every lane ends with the same total)
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            float v = acc[r][t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[r][t] = v;
        }

    if (wpt == 1) {
        if (r0 < g.rows) {
#pragma unroll
            for (int r = 0; r < kRows; ++r)
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (lane == (uint32_t)(r * MT + t) && r0 + r < g.rows && t0 + t < a.m)
                        g.Y[(size_t)(t0 + t) * g.ldy + r0 + r] = acc[r][t];
        }
        return;
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) red[warp][r * MT + t] = acc[r][t];
    }
    __syncthreads();
    if (part == 0 && r0 < g.rows && lane < (uint32_t)(kRows * MT)) {
        const uint32_t r = lane / MT, t = lane % MT;
        float v = red[warp][lane];
        for (uint32_t p = 1; p < wpt; ++p) v += red[warp + p][lane];
        if (r0 + r < g.rows && t0 + t < a.m) g.Y[(size_t)(t0 + t) * g.ldy + r0 + r] = v;
    }
}

// Any shape, any alignment: one warp per (row, token), lanes over k, one
// value per lane per step.  Used only when cols is not a multiple of the
// 16-byte vector or an activation row is not 16-byte aligned (the odd
// shapes of the reference's known-answer tests, e.g. 3x5 and 129x129).
template <int KIND>
__global__ void __launch_bounds__(kThreads) gemv_any_kernel(const __grid_constant__ Args a)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t item = (uint64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
    // item enumerates (segment row, token) pairs: rows of all segments, then tokens
    uint32_t total_rows = 0;
    for (int s = 0; s < a.nseg; ++s) total_rows += a.seg[s].rows;
    if (item >= (uint64_t)total_rows * a.m) return;
    uint32_t t = (uint32_t)(item / total_rows);
    uint32_t gr = (uint32_t)(item % total_rows);
    int s = 0;
    while (gr >= a.seg[s].rows) { gr -= a.seg[s].rows; ++s; }
    const GemvSeg &g = a.seg[s];
    const float *x = a.X + (size_t)t * a.ldx;
    float acc = 0.f;
    if constexpr (KIND == 0) {
        const uint8_t *wr = g.W + (size_t)gr * a.K;
        const float *sr = g.S + (size_t)(gr >> 7) * a.kblocks;
        for (uint32_t k = lane; k < a.K; k += 32) {
            uint32_t h;
            const uint32_t b = wr[k];
            asm("{\n\t.reg .b16 lo;\n\tcvt.u16.u32 lo, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, lo;\n\t}" : "=r"(h) : "r"(b));
            const float wv = __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
            acc = fmaf(wv * sr[k >> 7], x[k], acc);
        }
    } else {
        const uint16_t *wr = reinterpret_cast<const uint16_t *>(g.W) + (size_t)gr * a.K;
        for (uint32_t k = lane; k < a.K; k += 32)
            acc = fmaf(__uint_as_float((uint32_t)wr[k] << 16), x[k], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) g.Y[(size_t)t * g.ldy + gr] = acc;
}

__global__ void swiglu_kernel(const float *g, const float *u, float *o, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float v = g[i];
        o[i] = v / (1.0f + expf(-v)) * u[i];
    }
}

}  // namespace

uint32_t gemv_wpt(uint32_t rows, uint32_t K, int sms)
{
    const uint32_t tasks = (rows + kRows - 1) / kRows;
    const uint32_t nchunks = (K + 511) / 512;
    const uint64_t want = (uint64_t)sms * 24;  // warps that keep HBM busy
    uint32_t wpt = 1;
    while (wpt < 8 && (uint64_t)tasks * wpt < want && wpt * 2 <= nchunks) wpt *= 2;
    return wpt;
}

int launch_gemv(int kind, const GemvSeg *segs_in, int nseg, const float *X,
                uint32_t K, uint32_t ldx, uint32_t m, cudaStream_t st)
{
    if (nseg < 1 || nseg > 4 || m == 0 || K == 0) return set_error(Q35CU_ERR_ARG, "gemv: bad launch shape");
    Args a{};
    a.X = X;
    a.K = K;
    a.ldx = ldx;
    a.m = m;
    a.kblocks = (K + 127) / 128;
    a.nseg = nseg;
    const uint32_t per = kind == 0 ? 16 : 8;
    const bool vec_ok = (K % per == 0) && (ldx % 4 == 0) && ((uintptr_t)X % 16 == 0);
    uint32_t total_rows = 0;
    for (int s = 0; s < nseg; ++s) {
        a.seg[s] = segs_in[s];
        total_rows += segs_in[s].rows;
        if (((uintptr_t)segs_in[s].W % 16) != 0) return set_error(Q35CU_ERR_ARG, "gemv: weight not 16-byte aligned");
    }
    if (vec_ok) {
        const int sms = device_sms();
        uint32_t cta = 0;
        for (int s = 0; s < nseg; ++s) {
            const uint32_t wpt = gemv_wpt(a.seg[s].rows, K, sms);
            const uint32_t tasks = (a.seg[s].rows + kRows - 1) / kRows;
            a.seg[s].wpt = wpt;
            a.seg[s].cta_begin = cta;
            cta += (tasks * wpt + kWarps - 1) / kWarps;
        }
        const int mt = m == 1 ? 1 : (m == 2 ? 2 : 4);
        dim3 grid(cta, (m + mt - 1) / mt);
        if (grid.y > 65535) return set_error(Q35CU_ERR_ARG, "gemv: too many tokens (%u)", m);
        if (kind == 0) {
            if (mt == 1) gemv_vec_kernel<0, 1><<<grid, kThreads, 0, st>>>(a);
            else if (mt == 2) gemv_vec_kernel<0, 2><<<grid, kThreads, 0, st>>>(a);
            else gemv_vec_kernel<0, 4><<<grid, kThreads, 0, st>>>(a);
        } else {
            if (mt == 1) gemv_vec_kernel<1, 1><<<grid, kThreads, 0, st>>>(a);
            else if (mt == 2) gemv_vec_kernel<1, 2><<<grid, kThreads, 0, st>>>(a);
            else gemv_vec_kernel<1, 4><<<grid, kThreads, 0, st>>>(a);
        }
    } else {
        const uint64_t items = (uint64_t)total_rows * m;
        const uint64_t blocks = (items + kWarps - 1) / kWarps;
        if (blocks > 0x7FFFFFFFull) return set_error(Q35CU_ERR_ARG, "gemv: shape too large for the generic kernel");
        if (kind == 0) gemv_any_kernel<0><<<(unsigned)blocks, kThreads, 0, st>>>(a);
        else gemv_any_kernel<1><<<(unsigned)blocks, kThreads, 0, st>>>(a);
    }
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

int launch_swiglu(const float *g, const float *u, float *o, size_t n, cudaStream_t st)
{
    const int sms = device_sms();
    size_t blocks = (n + 255) / 256;
    if (blocks > (size_t)sms * 8) blocks = (size_t)sms * 8;
    if (blocks == 0) return Q35CU_OK;
    swiglu_kernel<<<(unsigned)blocks, 256, 0, st>>>(g, u, o, n);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

}  // namespace q35cu
