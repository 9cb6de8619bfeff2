// Tensor-core prefill GEMM (M >= 128 tokens), sm_100a: TMA + tcgen05 + TMEM.
//
// Replaces the CPU loop of q35_mm_fp8_batch (qwen35-c/src/q35_mm.c:158-172)
// for prefill-sized batches.  Y[t, n] = sum_k Xb[t, k] * e4m3(W[n, k]) * s[n/128, k/128]
// with the activations Xb rounded to bf16 (the prefill contract: relative
// L2 error <= 5e-3 against the reference on the same bf16-valued X).
//
// Roofline: tensor cores.  2*M*N*K flops per launch.
//
// One CTA computes a 128 (weight rows) x 128 (tokens) tile over all of K:
//   warp 0      TMA producer: per 128-column block kb, the fp8 weight tile
//               [128 rows x 128 B] and the bf16 activation tile [128 tokens x
//               128 cols] (two 64-column boxes), both 128B-swizzled, into a
//               3-stage ring (mbarrier complete_tx);
//   warps 2-9   converters: two threads per row turn the fp8 tile into bf16 --
//               exact (e4m3 -> f16 -> f32 -> bf16 loses nothing) -- written in
//               the canonical K-major 128B-swizzle layout the MMA reads
//               (two 64-column atoms), double-buffered, then a proxy fence;
//   warp 1      one elected thread issues tcgen05.mma kind::f16 (A = the
//               bf16 weight tile, M = 128; B = the activation tile, N = 128;
//               8 steps of K = 16) into a fresh TMEM partial P[kb % 2];
//   warps 10-13 epilogue: each thread owns one weight row (a TMEM lane) and
//               promotes  ACC += s[n/128, kb] * P  for its 128 token columns
//               (ACC also in TMEM), then stores Y from the last block.
// TMEM: P0 | P1 | ACC = 384 of 512 columns.  The per-128-K promotion keeps
// the block scale out of the MMA operands, so the weight operand stays
// exact and the scale is applied once per block in fp32.
//
// Every mbarrier wait is bounded; a wait that gives up records
// Q35CU_ERR_TIMEOUT in the GEMM's device status word and the CTA winds down
// (the producer waits, bounded, for its copies in flight; TMEM is freed).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "q35cu_internal.h"

namespace q35cu {

__device__ uint32_t g_gemm_status;

namespace {

constexpr int kBM = 128;   // weight rows per tile (MMA M)
constexpr int kBN = 128;   // tokens per tile (MMA N)
constexpr int kBK = 128;   // columns per block (one scale block)
constexpr int kStages = 3;
constexpr uint32_t kXTile = kBN * kBK * 2;  // 32 KB bf16
constexpr uint32_t kWTile = kBM * kBK;      // 16 KB fp8
constexpr uint32_t kATile = kBM * kBK * 2;  // 32 KB bf16
constexpr uint32_t kAtom = 128 * 128;       // one 64-column swizzle atom of 128 rows
constexpr uint32_t kSpin = 1u << 22;
constexpr int kConvWarps = 8;   // fp8 -> bf16 converters (two threads per weight row)
constexpr int kThreads = (2 + kConvWarps + 4) * 32;

struct GemmArgs {
    const float *S;  // scales [ceil(N/128), kblocks]
    float *Y;        // [m, N] token-major
    uint32_t N, K, m, kblocks;
};

struct Smem {  // offsets from the 1024-aligned base
    static constexpr uint32_t x(int s) { return s * (kXTile + kWTile); }
    static constexpr uint32_t w(int s) { return s * (kXTile + kWTile) + kXTile; }
    static constexpr uint32_t a(int j) { return kStages * (kXTile + kWTile) + j * kATile; }
    static constexpr uint32_t bars = kStages * (kXTile + kWTile) + 2 * kATile;
    static constexpr uint32_t total = bars + 256;
};

__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t n)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity)
{
    for (uint32_t i = 0; i < kSpin; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(sa(b)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    atomicExch(&g_gemm_status, (uint32_t)Q35CU_ERR_TIMEOUT);
    return false;
}

__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(sa(dst)), "l"(map), "r"(c0), "r"(c1), "r"(sa(bar))
        : "memory");
}

// UMMA shared-memory descriptor: K-major, 128B swizzle, 8-row core groups 1024 B apart
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;              // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;              // descriptor version for tcgen05
    d |= (uint64_t)2 << 61;              // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: D f32, A bf16, B bf16, both K-major, M = 128, N = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// four e4m3 bytes -> four bf16, exact (e4m3 -> f16 -> f32 -> bf16 only widens)
__device__ __forceinline__ uint2 e4m3x4_to_bf16x4(uint32_t w)
{
    uint32_t h01, h23;
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(h01), "=r"(h23)
        : "r"(w));
    const float2 f01 = __half22float2(*reinterpret_cast<__half2 *>(&h01));
    const float2 f23 = __half22float2(*reinterpret_cast<__half2 *>(&h23));
    uint2 r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r.x) : "f"(f01.y), "f"(f01.x));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r.y) : "f"(f23.y), "f"(f23.x));
    return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                       const __grid_constant__ GemmArgs a)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Smem::bars);  // [3] TMA -> converters, MMA
    uint64_t *empty = full + kStages;                                 // [3] converters + MMA -> TMA
    uint64_t *a_full = empty + kStages;                               // [2] converters -> MMA
    uint64_t *a_empty = a_full + 2;                                   // [2] MMA -> converters
    uint64_t *p_full = a_empty + 2;                                   // [2] MMA -> epilogue
    uint64_t *p_empty = p_full + 2;                                   // [2] epilogue -> MMA
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(p_empty + 2);

    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t n0 = blockIdx.x * kBM, m0 = blockIdx.y * kBN;
    const uint32_t nkb = a.kblocks;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sa(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (t == 32) {
        for (int i = 0; i < kStages; ++i) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], kConvWarps + 1);
        }
        for (int i = 0; i < 2; ++i) {
            bar_init(&a_full[i], kConvWarps);
            bar_init(&a_empty[i], 1);
            bar_init(&p_full[i], 1);
            bar_init(&p_empty[i], 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer -------------------------------------
        if (lane == 0) {
            uint32_t issued = 0;
            bool ok = true;
            for (uint32_t kb = 0; kb < nkb && ok; ++kb, ++issued) {
                const int s = kb % kStages;
                if (kb >= kStages) ok = bar_wait(&empty[s], ((kb / kStages) - 1) & 1);
                if (!ok) break;
                bar_expect(&full[s], kXTile + kWTile);
                tma_2d(sm + Smem::x(s), &map_x, (int)(kb * kBK), (int)m0, &full[s]);
                tma_2d(sm + Smem::x(s) + kAtom, &map_x, (int)(kb * kBK + 64), (int)m0, &full[s]);
                tma_2d(sm + Smem::w(s), &map_w, (int)(kb * kBK), (int)n0, &full[s]);
            }
            for (uint32_t i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
                bar_wait(&full[i % kStages], (i / kStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ---------------------------------------
        if (lane == 0) {
            bool ok = true;
            for (uint32_t kb = 0; kb < nkb && ok; ++kb) {
                const int s = kb % kStages, j = kb % 2;
                ok = bar_wait(&full[s], (kb / kStages) & 1) && bar_wait(&a_full[j], (kb / 2) & 1);
                if (ok && kb >= 2) ok = bar_wait(&p_empty[j], ((kb / 2) - 1) & 1);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t abase = sa(sm + Smem::a(j)), xbase = sa(sm + Smem::x(s));
                const uint32_t d = tmem + j * kBN;
#pragma unroll
                for (int ks = 0; ks < kBK / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * kAtom + (ks & 3) * 32;
                    mma_bf16(d, sw128_desc(abase + off), sw128_desc(xbase + off), ks > 0);
                }
                mma_commit(&p_full[j]);
                mma_commit(&empty[s]);
                mma_commit(&a_empty[j]);
            }
            // the last partial must have landed before the CTA can free TMEM
            if (ok && nkb) bar_wait(&p_full[(nkb - 1) % 2], ((nkb - 1) / 2) & 1);
        }
    } else if (warp < 2 + kConvWarps) {
        // ---------------- converters: fp8 -> bf16, swizzled -----------------
        const uint32_t r = (t - 64) >> 1;        // weight row of the tile
        const int c0 = ((t - 64) & 1) * 4;       // this thread's four 16-byte chunks
        bool ok = true;
        for (uint32_t kb = 0; kb < nkb && ok; ++kb) {
            const int s = kb % kStages, j = kb % 2;
            ok = bar_wait(&full[s], (kb / kStages) & 1);
            if (ok && kb >= 2) ok = bar_wait(&a_empty[j], ((kb / 2) - 1) & 1);
            if (!ok) break;
            const uint8_t *wrow = sm + Smem::w(s) + r * 128;
            uint8_t *arow = sm + Smem::a(j) + r * 128;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int c = c0 + cc;
                const uint4 v = *reinterpret_cast<const uint4 *>(wrow + ((c ^ (r & 7)) << 4));
                const uint2 b0 = e4m3x4_to_bf16x4(v.x), b1 = e4m3x4_to_bf16x4(v.y);
                const uint2 b2 = e4m3x4_to_bf16x4(v.z), b3 = e4m3x4_to_bf16x4(v.w);
                // bf16 chunks 2c and 2c+1 of the 16 in this row: atom (2c)/8, chunk (2c)%8
                const uint32_t q0 = 2 * c, q1 = 2 * c + 1;
                *reinterpret_cast<uint4 *>(arow + (q0 >> 3) * kAtom + (((q0 & 7) ^ (r & 7)) << 4)) =
                    make_uint4(b0.x, b0.y, b1.x, b1.y);
                *reinterpret_cast<uint4 *>(arow + (q1 >> 3) * kAtom + (((q1 & 7) ^ (r & 7)) << 4)) =
                    make_uint4(b2.x, b2.y, b3.x, b3.y);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                bar_arrive(&a_full[j]);
                bar_arrive(&empty[s]);
            }
        }
    } else {
        // ---------------- epilogue: promotion and store -----------------------
        const uint32_t quad = warp & 3;                 // TMEM lanes this warp may touch
        const uint32_t row = quad * 32 + lane;          // weight row of the tile
        const uint32_t n = n0 + row;
        const uint32_t sb = (n0 / 128 < (a.N + 127) / 128) ? n0 / 128 : 0;
        const float *srow = a.S + (size_t)sb * nkb;
        const uint32_t lane_base = tmem + ((quad * 32) << 16);
        bool ok = true;
        for (uint32_t kb = 0; kb < nkb && ok; ++kb) {
            const int j = kb % 2;
            ok = bar_wait(&p_full[j], (kb / 2) & 1);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const float sc = __ldg(srow + kb);
            const bool last = kb + 1 == nkb;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t p[32], q[32];
                tmem_ld32(lane_base + j * kBN + c * 32, p);
                if (kb) tmem_ld32(lane_base + 2 * kBN + c * 32, q);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float acc = kb ? fmaf(sc, __uint_as_float(p[i]), __uint_as_float(q[i]))
                                         : sc * __uint_as_float(p[i]);
                    q[i] = __float_as_uint(acc);
                }
                if (!last) {
                    tmem_st32(lane_base + 2 * kBN + c * 32, q);
                } else if (n < a.N) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const uint32_t mm = m0 + c * 32 + i;
                        if (mm < a.m) a.Y[(size_t)mm * a.N + n] = __uint_as_float(q[i]);
                    }
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) bar_arrive(&p_empty[j]);
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

// bf16 rounding of fp32 activations (nearest even)
__global__ void f32_to_bf16_rows(const float *x, uint16_t *y, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __bfloat16_as_ushort(__float2bfloat16_rn(x[i]));
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder()
{
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

int make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer)
{
    EncodeTiled enc = encoder();
    if (!enc) return set_error(Q35CU_ERR_CUDA, "cuTensorMapEncodeTiled not available");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(Q35CU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return Q35CU_OK;
}

}  // namespace

int launch_gemm_fp8(const q35cu_weight *w, const uint16_t *Xb, uint32_t m, float *Y, cudaStream_t st)
{
    const uint32_t N = w->rows, K = w->cols;
    if (K % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: cols %u not a multiple of 16", K);
    if (((uintptr_t)Xb % 16) || ((uintptr_t)w->d_w % 16)) return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned operand");
    if ((N + kBM - 1) / kBM > 0x7FFFFFFFu || (m + kBN - 1) / kBN > 65535u)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8: shape too large");
    CUtensorMap mx, mw;
    int rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, Xb, K, m, (uint64_t)K * 2, 64, kBN);
    if (rc) return rc;
    rc = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->d_w, K, N, K, 128, kBM);
    if (rc) return rc;
    GemmArgs a{w->d_s, Y, N, K, m, (K + kBK - 1) / kBK};
    static bool configured[64] = {};
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    const size_t smem = Smem::total + 1024;
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(gemm_fp8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured[dev] = true;
    }
    const dim3 grid((N + kBM - 1) / kBM, (m + kBN - 1) / kBN);
    gemm_fp8_tc_kernel<<<grid, kThreads, smem, st>>>(mx, mw, a);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

int launch_round_bf16(const float *x, uint16_t *y, size_t n, cudaStream_t st)
{
    if (!n) return Q35CU_OK;
    size_t blocks = (n + 255) / 256;
    const size_t cap = (size_t)device_sms() * 16;
    if (blocks > cap) blocks = cap;
    f32_to_bf16_rows<<<(unsigned)blocks, 256, 0, st>>>(x, y, n);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

// ---------------------------------------------------------------------------
// Prefill GEMM for callers that must not allocate device memory.
//
// q35cu_gemm_fp8 takes bf16 activations; a caller holding fp32 activations
// needs a bf16 copy first, and the host entry point q35_mm_fp8_batch keeps
// that copy in a buffer it allocates.  Some callers cannot let the library
// call cudaMalloc at that point: a serving process that reserved its whole
// HBM budget up front, or a decode/prefill loop that cannot afford the
// device-wide synchronisation a cudaMalloc/cudaFree may imply.  For them the
// bf16 copy lives in a fixed array compiled into this file instead.
//
//   * the array holds kNoAllocMaxActs bf16 values (16 MiB); every GPU that
//     loads the library keeps it until the process exits;
//   * a call with m * cols > kNoAllocMaxActs is rejected with Q35CU_ERR_ARG;
//   * every call reuses the same array: two calls whose work overlaps on the
//     GPU (different streams, no ordering) race on it;
//   * each call overwrites exactly the m * cols values it reads, so nothing
//     needs clearing between calls;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) and sets the GEMM's shared-memory limit; make
//     that first call before any stream capture.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocMaxActs = (size_t)8 << 20;
static __device__ __align__(256) uint16_t g_noalloc_acts[kNoAllocMaxActs];

namespace {

__global__ void round_bf16_noalloc(const float *x, uint16_t *y, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __bfloat16_as_ushort(__float2bfloat16_rn(x[i]));
}

// the array's device address, looked up once per device with that device current
int noalloc_scratch(uint16_t **out)
{
    static uint16_t *addr[64] = {};
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    if (!addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_acts);
        if (e != cudaSuccess || !p) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_acts)");
        addr[dev] = static_cast<uint16_t *>(p);
    }
    *out = addr[dev];
    return Q35CU_OK;
}

}  // namespace

int gemm_fp8_f32_noalloc(const q35cu_weight *w, const float *X, uint32_t m, float *Y, cudaStream_t st)
{
    if (!w || w->kind != 0 || !X || !Y) return set_error(Q35CU_ERR_ARG, "gemm_fp8_f32_noalloc: bad arguments");
    if (!m) return Q35CU_OK;
    const size_t n = (size_t)m * w->cols;
    if (n > kNoAllocMaxActs)
        return set_error(Q35CU_ERR_ARG,
                         "gemm_fp8_f32_noalloc: %u tokens x %u cols = %zu activations exceed the fixed %zu-value "
                         "scratch; split the batch",
                         m, w->cols, n, kNoAllocMaxActs);
    uint16_t *xbf = nullptr;
    int rc = noalloc_scratch(&xbf);
    if (rc) return rc;
    int dev = 0, sms = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    Q35CU_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    size_t blocks = (n + 255) / 256;
    if (blocks > (size_t)sms * 16) blocks = (size_t)sms * 16;
    round_bf16_noalloc<<<(unsigned)blocks, 256, 0, st>>>(X, xbf, n);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return launch_gemm_fp8(w, xbf, m, Y, st);
}

int gemm_status(uint32_t *status, bool clear)
{
    Q35CU_CUDA(cudaMemcpyFromSymbol(status, g_gemm_status, 4));
    if (clear) {
        const uint32_t z = 0;
        Q35CU_CUDA(cudaMemcpyToSymbol(g_gemm_status, &z, 4));
    }
    return Q35CU_OK;
}

}  // namespace q35cu

// The allocation-free prefill entry point (see gemm_fp8_f32_noalloc above).
// `stream` NULL means the legacy default stream.
extern "C" __attribute__((visibility("default"))) int q35cu_gemm_fp8_f32_noalloc(const q35cu_weight *w,
                                                                               const float *X, uint32_t m,
                                                                               float *Y, void *stream)
{
    return q35cu::gemm_fp8_f32_noalloc(w, X, m, Y, static_cast<cudaStream_t>(stream));
}
