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
// Decomposition ("row stream"):
//   * one CTA per SM; CTA c owns the contiguous virtual rows
//     [c*R/G, (c+1)*R/G) of the launch (R = rows of all segments, G = grid),
//     so every SM streams the same number of bytes (no partial waves);
//   * thread t owns a fixed K-slice: 16 bytes (one 16-byte vector) per pass
//     at k = p*T*16 + t*16, with T = blockDim.x and P = ceil(K/16/T) passes,
//     T and P a function of K only.  Its activation slice x[k..k+16) stays
//     in registers for the whole kernel when P == 1;
//   * rows stream through a double-buffered register pipeline in groups of
//     GR rows: the next group's 16-byte loads (and block scales) are issued
//     before the current group is converted and multiplied, across block,
//     pass and segment boundaries;
//   * per row and pass the thread forms d = sum_{j<16} w_j x_j and folds
//     part_r = fma(s[r/128, k/128], d, part_r);
//   * every 32/MT rows the 32 x 32 partials of a warp are reduced with a
//     transpose butterfly (31 shuffles; the same association as a plain xor
//     butterfly), warps are summed in fixed order through shared memory and
//     one thread per (row, token) writes Y.
// The per-row arithmetic is therefore independent of m, of the token tile
// width and of the other weights sharing a launch: batch, multi and single
// calls agree bit for bit (the contract of qwen35-c/tests/test_batch_mm.c),
// and repeated runs are identical (no atomics).
//
// e4m3 decoding.  The hardware unpack (cvt.rn.{f16x2,bf16x2}.e4m3x2) runs on
// the quarter-rate XU pipe, which would cap the kernel below HBM speed if it
// decoded every byte.  Variant CONV splits each vector: half through the
// hardware unpack, half through an ALU bit transform that places the 7
// exponent+mantissa bits of e4m3 under an f16 exponent (value * 2^-8 exactly,
// subnormals included; the 2^8 is restored by one exact fma per vector).  The
// bit transform maps the NaN codes 0x7F/0xFF to finite values, so a weight
// in which the upload scan found a NaN code takes a checked path that turns
// the affected dot products into NaN, as the reference's LUT does.
//
// Programmatic dependent launch: the kernel triggers its dependents at
// entry and issues its first weight loads before griddepcontrol.wait, so in
// a chain of projections the next kernel's weight stream starts while the
// previous kernel drains.  Nothing is written and no activation is read
// before the wait.
#include <cuda_fp16.h>

#include <type_traits>

#include "q35cu_internal.h"

namespace q35cu {
namespace {

constexpr int kMaxThreads = 384;
constexpr int kMaxWarps = kMaxThreads / 32;
constexpr uint32_t kFull = 0xffffffffu;

struct Seg {
    const uint8_t *W;
    const float *S;
    float *Y;
    uint32_t rows, ldy, vbegin;  // vbegin: first virtual row of the segment
    uint32_t has_nan;            // weight holds e4m3 NaN codes (0x7F / 0xFF)
};

struct Args {
    Seg seg[4];
    const float *X;
    uint32_t K, ldx, m, kblocks, total_rows, passes;
    int nseg;
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ uint4 ld_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---- e4m3 decoding -------------------------------------------------------
// hardware: bytes (b1 b0) of the low half -> f16x2 (b0 low), exact
__device__ __forceinline__ void hw_f16x2(uint32_t w, uint32_t &lo, uint32_t &hi)
{
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}
// ALU: f16x2 holding value * 2^-8 of bytes b0 (low) and b1 (high) of
// h = [b1 0 b0 0] (a prmt of the word); sign to bit 15, E and M under the
// f16 exponent/mantissa: exact for normals and subnormals alike.
__device__ __forceinline__ uint32_t bt_f16x2(uint32_t h)
{
    return ((h & 0x7F007F00u) >> 1) | (h & 0x80008000u);
}
__device__ __forceinline__ float2 h2f(uint32_t h)
{
    return __half22float2(*reinterpret_cast<__half2 *>(&h));
}

__device__ __forceinline__ unsigned long long pk(float a, float b)
{
    return (unsigned long long)__float_as_uint(a) | ((unsigned long long)__float_as_uint(b) << 32);
}
__device__ __forceinline__ void fma2(unsigned long long &acc, float w0, float w1, float x0, float x1)
{
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(pk(w0, w1)), "l"(pk(x0, x1)));
}
__device__ __forceinline__ float hsum2(unsigned long long v)
{
    return __uint_as_float((uint32_t)v) + __uint_as_float((uint32_t)(v >> 32));
}

// any byte of w equal to 0x7F or 0xFF
__device__ __forceinline__ bool nan_code(uint32_t w)
{
    return __vcmpeq4(w | 0x80808080u, 0xFFFFFFFFu) != 0u;
}

// dot of one 16-byte fp8 vector with x[16]
template <int CONV>
__device__ __forceinline__ float dot_fp8(const uint4 &v, const float *x, bool check_nan)
{
    unsigned long long a = 0ull, b = 0ull;
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
    if constexpr (CONV == 0) {  // all hardware
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t lo, hi;
            hw_f16x2(wd[q], lo, hi);
            const float2 f0 = h2f(lo), f1 = h2f(hi);
            fma2(q < 2 ? a : b, f0.x, f0.y, x[4 * q], x[4 * q + 1]);
            fma2(q < 2 ? a : b, f1.x, f1.y, x[4 * q + 2], x[4 * q + 3]);
        }
        return hsum2(a) + hsum2(b);
    } else {  // words 0,1 hardware, words 2,3 bit transform (x 2^-8)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            uint32_t lo, hi;
            hw_f16x2(wd[q], lo, hi);
            const float2 f0 = h2f(lo), f1 = h2f(hi);
            fma2(a, f0.x, f0.y, x[4 * q], x[4 * q + 1]);
            fma2(a, f1.x, f1.y, x[4 * q + 2], x[4 * q + 3]);
        }
#pragma unroll
        for (int q = 2; q < 4; ++q) {
            const float2 f0 = h2f(bt_f16x2(__byte_perm(wd[q], 0u, 0x1404)));
            const float2 f1 = h2f(bt_f16x2(__byte_perm(wd[q], 0u, 0x3424)));
            fma2(b, f0.x, f0.y, x[4 * q], x[4 * q + 1]);
            fma2(b, f1.x, f1.y, x[4 * q + 2], x[4 * q + 3]);
        }
        float d = fmaf(256.0f, hsum2(b), hsum2(a));
        if (check_nan && (nan_code(v.z) || nan_code(v.w))) d = __int_as_float(0x7fffffff);
        return d;
    }
}

__device__ __forceinline__ float dot_bf16(const uint4 &v, const float *x)
{
    unsigned long long a = 0ull;
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q)
        fma2(a, __uint_as_float(wd[q] << 16), __uint_as_float(wd[q] & 0xFFFF0000u), x[2 * q], x[2 * q + 1]);
    return hsum2(a);
}

// 32 values per lane -> lane j holds the warp total of slot j
__device__ __forceinline__ float transpose_reduce(float (&v)[32], uint32_t lane)
{
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
        const bool up = lane & w;
#pragma unroll
        for (int i = 0; i < w; ++i) {
            const float send = up ? v[i] : v[i + w];
            const float keep = up ? v[i + w] : v[i];
            v[i] = keep + __shfl_xor_sync(kFull, send, w);
        }
    }
    return v[0];
}

// position of one row group in the CTA's walk over (block, pass, group)
struct Pos {
    uint32_t b0, b1;  // block: virtual rows [b0, b1)
    uint32_t p, g;    // pass, group index inside the block
    int s;            // segment
    bool ok;
};

template <int KIND, int CONV, int MT, int GR>
__global__ void __launch_bounds__(kMaxThreads, 1) gemv_rs_kernel(const __grid_constant__ Args a)
{
    constexpr uint32_t EPV = KIND == 0 ? 16 : 8;  // values per 16-byte vector
    constexpr uint32_t ESZ = KIND == 0 ? 1 : 2;
    constexpr int BR = 32 / MT;                   // rows per reduction block
    constexpr int NG = BR / GR;                   // groups per (block, pass)
    static_assert(BR % GR == 0, "group must divide block");
    __shared__ float red[kMaxWarps][32];

    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
    const uint32_t T = blockDim.x, K = a.K, P = a.passes;
    const uint32_t tok0 = blockIdx.y * MT;
    const uint32_t vr0 = (uint32_t)(((uint64_t)blockIdx.x * a.total_rows) / gridDim.x);
    const uint32_t vr1 = (uint32_t)(((uint64_t)(blockIdx.x + 1) * a.total_rows) / gridDim.x);

    griddep_launch();

    auto seg_of = [&](uint32_t vr) {
        int s = 0;
#pragma unroll
        for (int i = 1; i < 4; ++i)
            if (i < a.nseg && vr >= a.seg[i].vbegin) s = i;
        return s;
    };
    auto block_at = [&](uint32_t vr) {
        Pos q;
        q.ok = vr < vr1;
        q.b0 = vr;
        q.s = q.ok ? seg_of(vr) : 0;
        const uint32_t send = a.seg[q.s].vbegin + a.seg[q.s].rows;
        uint32_t e = vr + BR;
        e = e < vr1 ? e : vr1;
        q.b1 = e < send ? e : send;
        q.p = 0;
        q.g = 0;
        return q;
    };
    auto advance = [&](Pos q) {
        if (q.g + 1 < (uint32_t)NG && q.b0 + (q.g + 1) * GR < q.b1) { q.g++; return q; }
        if (q.p + 1 < P) { q.p++; q.g = 0; return q; }
        return block_at(q.b1);
    };
    auto kpos = [&](uint32_t p) { return p * T * EPV + t * EPV; };

    uint4 wb[2][GR];
    float sb[2][GR];
    // B: buffer index as a compile-time constant, so wb/sb stay in registers
    auto load = [&](auto B, const Pos &q) {
        constexpr int b = decltype(B)::value;
        const Seg &sg = a.seg[q.s];
        const uint32_t k = kpos(q.p);
        const bool kv = k < K;
        const uint32_t kb = k >> 7;
#pragma unroll
        for (int i = 0; i < GR; ++i) {
            const uint32_t vr = q.b0 + q.g * GR + i;
            const bool v = kv && vr < q.b1;
            const uint32_t r = vr - sg.vbegin;
            wb[b][i] = v ? ld_stream(sg.W + ((size_t)r * K + k) * ESZ) : make_uint4(0, 0, 0, 0);
            if constexpr (KIND == 0) sb[b][i] = v ? __ldg(sg.S + (size_t)(r >> 7) * a.kblocks + kb) : 0.f;
        }
    };

    float xr[MT][EPV];
    auto load_x = [&](uint32_t p) {
        const uint32_t k = kpos(p);
#pragma unroll
        for (int tt = 0; tt < MT; ++tt) {
            const bool v = k < K && tok0 + tt < a.m;
            const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)(tok0 + tt) * a.ldx + k);
#pragma unroll
            for (int q = 0; q < (int)EPV / 4; ++q) {
                const float4 f = v ? __ldg(xp + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                xr[tt][4 * q] = f.x; xr[tt][4 * q + 1] = f.y; xr[tt][4 * q + 2] = f.z; xr[tt][4 * q + 3] = f.w;
            }
        }
    };

    float part[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) part[i] = 0.f;

    // one group: prefetch the next group into the other buffer, multiply the
    // current one, close the block when it ends.  Returns the next position.
    auto step = [&](auto B, const Pos &cur) {
        constexpr int b = decltype(B)::value;
        const Pos nx = advance(cur);
        if (nx.ok) load(std::integral_constant<int, b ^ 1>{}, nx);
        const bool chk = KIND == 0 && a.seg[cur.s].has_nan;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            if (cur.g == (uint32_t)g) {
#pragma unroll
                for (int i = 0; i < GR; ++i) {
#pragma unroll
                    for (int tt = 0; tt < MT; ++tt) {
                        float &pr = part[(g * GR + i) * MT + tt];
                        if constexpr (KIND == 0) pr = fmaf(sb[b][i], dot_fp8<CONV>(wb[b][i], xr[tt], chk), pr);
                        else pr += dot_bf16(wb[b][i], xr[tt]);
                    }
                }
            }
        }
        if (!nx.ok || nx.b0 != cur.b0) {  // block complete: reduce and store
            const float v = transpose_reduce(part, lane);
            red[warp][lane] = v;
            __syncthreads();
            if (warp == 0) {
                float acc = red[0][lane];
                for (uint32_t w = 1; w < nw; ++w) acc += red[w][lane];
                const uint32_t vr = cur.b0 + lane / MT, tt = lane % MT;
                const Seg &sg = a.seg[cur.s];
                if (vr < cur.b1 && tok0 + tt < a.m) sg.Y[(size_t)(tok0 + tt) * sg.ldy + (vr - sg.vbegin)] = acc;
            }
            __syncthreads();
#pragma unroll
            for (int i = 0; i < 32; ++i) part[i] = 0.f;
        }
        if (nx.ok && P > 1 && nx.p != cur.p) load_x(nx.p);
        return nx;
    };

    Pos cur = block_at(vr0);
    if (cur.ok) load(std::integral_constant<int, 0>{}, cur);
    griddep_wait();  // activations of the previous kernel are visible from here on
    if (!cur.ok) return;
    load_x(0);
    while (true) {
        cur = step(std::integral_constant<int, 0>{}, cur);
        if (!cur.ok) break;
        cur = step(std::integral_constant<int, 1>{}, cur);
        if (!cur.ok) break;
    }
}

// Any shape, any alignment: one warp per (row, token), lanes over k, one
// value per lane per step.  Used only when cols is not a multiple of the
// 16-byte vector or an activation row is not 16-byte aligned (the odd
// shapes of the reference's known-answer tests, e.g. 3x5 and 129x129).
template <int KIND>
__global__ void __launch_bounds__(256) gemv_any_kernel(const __grid_constant__ Args a)
{
    griddep_launch();
    griddep_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t item = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= (uint64_t)a.total_rows * a.m) return;
    const uint32_t t = (uint32_t)(item / a.total_rows);
    uint32_t gr = (uint32_t)(item % a.total_rows);
    int s = 0;
    while (s + 1 < a.nseg && gr >= a.seg[s + 1].vbegin) ++s;
    const Seg &g = a.seg[s];
    gr -= g.vbegin;
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
        for (uint32_t k = lane; k < a.K; k += 32) acc = fmaf(__uint_as_float((uint32_t)wr[k] << 16), x[k], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
    if (lane == 0) g.Y[(size_t)t * g.ldy + gr] = acc;
}

__global__ void swiglu_kernel(const float *g, const float *u, float *o, size_t n)
{
    griddep_launch();
    griddep_wait();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = g[i];
        o[i] = v / (1.0f + expf(-v)) * u[i];
    }
}

// scan an FP8 weight for the NaN codes 0x7F / 0xFF
__global__ void nan_scan_kernel(const uint4 *w, size_t n16, const uint8_t *tail, uint32_t ntail, uint32_t *flag)
{
    bool found = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = w[i];
        found |= nan_code(v.x) | nan_code(v.y) | nan_code(v.z) | nan_code(v.w);
    }
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < ntail; i += blockDim.x) found |= (tail[i] & 0x7F) == 0x7F;
    if (__syncthreads_or(found) && threadIdx.x == 0) atomicOr(flag, 1u);
}

template <typename Kern>
int launch_pdl(Kern k, dim3 grid, dim3 block, cudaStream_t st, const Args &a)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35CU_CUDA(cudaLaunchKernelEx(&cfg, k, a));
    count_launch();
    return Q35CU_OK;
}

int conv_variant()
{
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("Q35CU_GEMV_CONV");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v;
}

template <int KIND, int CONV>
int launch_rs(const Args &a, uint32_t threads, dim3 grid, int mt, cudaStream_t st)
{
    if (mt == 1) return launch_pdl(gemv_rs_kernel<KIND, CONV, 1, 8>, grid, dim3(threads), st, a);
    if (mt == 2) return launch_pdl(gemv_rs_kernel<KIND, CONV, 2, 8>, grid, dim3(threads), st, a);
    return launch_pdl(gemv_rs_kernel<KIND, CONV, 4, 4>, grid, dim3(threads), st, a);
}

}  // namespace

// threads and passes of the row-stream kernel: a function of K only
void gemv_geometry(int kind, uint32_t K, uint32_t *threads, uint32_t *passes)
{
    const uint32_t epv = kind == 0 ? 16 : 8;
    const uint32_t nvec = (K + epv - 1) / epv;
    const uint32_t P = (nvec + kMaxThreads - 1) / kMaxThreads;
    uint32_t T = (nvec + P - 1) / P;
    T = (T + 31) / 32 * 32;
    *threads = T;
    *passes = P;
}

int launch_gemv(int kind, const GemvSeg *segs_in, int nseg, const float *X, uint32_t K, uint32_t ldx, uint32_t m,
                cudaStream_t st)
{
    if (nseg < 1 || nseg > 4 || m == 0 || K == 0) return set_error(Q35CU_ERR_ARG, "gemv: bad launch shape");
    Args a{};
    a.X = X;
    a.K = K;
    a.ldx = ldx;
    a.m = m;
    a.kblocks = (K + 127) / 128;
    a.nseg = nseg;
    const uint32_t epv = kind == 0 ? 16 : 8;
    bool vec_ok = (K % epv == 0) && (ldx % 4 == 0) && ((uintptr_t)X % 16 == 0);
    uint32_t vb = 0;
    for (int s = 0; s < nseg; ++s) {
        const GemvSeg &g = segs_in[s];
        a.seg[s] = Seg{g.W, g.S, g.Y, g.rows, g.ldy, vb, g.has_nan};
        vb += g.rows;
        if ((uintptr_t)g.W % 16) vec_ok = false;
    }
    a.total_rows = vb;
    if (vb == 0) return Q35CU_OK;
    if (vec_ok) {
        uint32_t T, P;
        gemv_geometry(kind, K, &T, &P);
        a.passes = P;
        const int mt = m == 1 ? 1 : (m == 2 ? 2 : 4);
        const uint32_t sms = (uint32_t)device_sms();
        const uint32_t gx = vb < sms ? vb : sms;
        const uint32_t gy = (m + mt - 1) / mt;
        if (gy > 65535) return set_error(Q35CU_ERR_ARG, "gemv: too many tokens (%u)", m);
        const dim3 grid(gx, gy);
        if (kind == 1) return launch_rs<1, 1>(a, T, grid, mt, st);
        return conv_variant() == 0 ? launch_rs<0, 0>(a, T, grid, mt, st) : launch_rs<0, 1>(a, T, grid, mt, st);
    }
    const uint64_t items = (uint64_t)vb * m;
    const uint64_t blocks = (items + 7) / 8;
    if (blocks > 0x7FFFFFFFull) return set_error(Q35CU_ERR_ARG, "gemv: shape too large for the generic kernel");
    if (kind == 0) return launch_pdl(gemv_any_kernel<0>, dim3((unsigned)blocks), dim3(256), st, a);
    return launch_pdl(gemv_any_kernel<1>, dim3((unsigned)blocks), dim3(256), st, a);
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

int scan_nan_codes(const uint8_t *W, size_t bytes, uint32_t *d_flag, cudaStream_t st, bool *has_nan)
{
    Q35CU_CUDA(cudaMemsetAsync(d_flag, 0, 4, st));
    const size_t n16 = bytes / 16;
    const uint32_t tail = (uint32_t)(bytes % 16);
    size_t blocks = (n16 + 255) / 256;
    const size_t cap = (size_t)device_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    nan_scan_kernel<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const uint4 *>(W), n16, W + n16 * 16, tail,
                                                      d_flag);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    uint32_t h = 0;
    Q35CU_CUDA(cudaMemcpyAsync(&h, d_flag, 4, cudaMemcpyDeviceToHost, st));
    Q35CU_CUDA(cudaStreamSynchronize(st));
    *has_nan = h != 0;
    return Q35CU_OK;
}

}  // namespace q35cu
