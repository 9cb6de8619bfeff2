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
// Decomposition (one CTA per SM, "row stream"):
//   * CTA c owns the contiguous virtual rows [c*R/G, (c+1)*R/G) of the launch
//     (R = rows of all segments, G = grid), so every SM streams the same
//     number of bytes and there is no partial wave;
//   * a producer warp streams those rows, a few whole rows per stage, into a
//     shared-memory ring with cp.async.bulk (TMA bulk copies completing on
//     mbarriers): memory-level parallelism comes from the copy engine, not
//     from registers, so the ring keeps ~100 KB per SM in flight;
//   * consumer thread t owns a fixed K-slice -- one 16-byte vector per pass
//     at k = p*T*16 + t*16 (T consumer threads, P = ceil(K/16/T) passes, both
//     a function of K only) -- and keeps x[k..k+16) of every pass and token
//     in registers for the whole kernel; it reads its vector of each staged
//     row from shared memory (a warp reads 512 contiguous bytes) and folds
//       part_r = fma(s[r/128, k/128], sum_{j<16} w_j x_j, part_r)
//     in pass order;
//   * every 32/MT rows the 32 x 32 partials of a warp are reduced with a
//     transpose butterfly (31 shuffles, the association of a plain xor
//     butterfly), the warps are summed in fixed order through shared memory
//     and one thread per (row, token) writes Y.
// The per-row arithmetic is therefore independent of m, of the token tile,
// of the ring geometry and of the other weights sharing a launch: batch,
// multi and single calls agree bit for bit (the contract of
// qwen35-c/tests/test_batch_mm.c), and repeated runs are identical.
//
// e4m3 decoding uses the hardware unpack cvt.rn.f16x2.e4m3x2 (exact; NaN
// codes stay NaN, as in the reference's LUT) and products run as packed
// fma.rn.f32x2: about two issued instructions per weight byte.
//
// Programmatic dependent launch: the kernel triggers its dependents at
// entry; the producer streams weights without waiting for the previous
// kernel, and only the consumers execute griddepcontrol.wait before they
// read activations, so in a chain of projections the next weight stream
// starts while the previous kernel drains.
//
// Every mbarrier wait is bounded.  A wait that gives up records
// Q35CU_ERR_TIMEOUT in the device status word (read by q35cu_device_status),
// and the CTA winds down: the producer stops issuing and waits, bounded, for
// the copies it has in flight before the CTA exits.
#include <cuda_fp16.h>

#include <cstring>
#include <type_traits>

#include "p2p_ll.cuh"
#include "q35cu_internal.h"

namespace q35cu {

// bounded device-side waits that gave up leave their code here
__device__ uint32_t g_device_status;

namespace {

constexpr int kMaxCons = 384;  // consumer threads per CTA
constexpr int kMaxWarps = kMaxCons / 32;
constexpr int kMaxStages = 8;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kFull = 0xffffffffu;
constexpr uint32_t kRingBudget = 200 * 1024;  // ring bytes per CTA (one CTA per SM)

struct Seg {
    const uint8_t *W;
    const float *S;
    float *Y;
    uint32_t rows, ldy, vbegin;  // vbegin: first virtual row of the segment
    uint32_t has_nan;
};

struct Args {
    Seg seg[4];
    const float *X;
    uint32_t K, ldx, m, kblocks, total_rows;
    uint32_t cons;         // consumer threads (multiple of 32)
    uint32_t stages;       // ring slots
    uint32_t slot_bytes;   // bytes of one ring slot (stage rows * row bytes)
    int nseg;
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte streaming load of read-only data (no L1 allocation, 256-byte L2 prefetch)
__device__ __forceinline__ uint4 ld_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait; false = gave up (status recorded)
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity)
{
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(b, parity)) return true;
    atomicExch(&g_device_status, (uint32_t)Q35CU_ERR_TIMEOUT);
    return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(saddr(dst)), "l"(src), "r"(bytes), "r"(saddr(bar))
                 : "memory");
}

// ---- decoding + dot products ---------------------------------------------
__device__ __forceinline__ void hw_f16x2(uint32_t w, uint32_t &lo, uint32_t &hi)
{
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}
__device__ __forceinline__ float2 h2f(uint32_t h) { return __half22float2(*reinterpret_cast<__half2 *>(&h)); }
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

// 16 e4m3 values . x[16]: two packed accumulators (even/odd pairs of words)
__device__ __forceinline__ float dot_fp8(const uint4 &v, const float *x)
{
    unsigned long long a = 0ull, b = 0ull;
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t lo, hi;
        hw_f16x2(wd[q], lo, hi);
        const float2 f0 = h2f(lo), f1 = h2f(hi);
        fma2(q & 1 ? b : a, f0.x, f0.y, x[4 * q], x[4 * q + 1]);
        fma2(q & 1 ? b : a, f1.x, f1.y, x[4 * q + 2], x[4 * q + 3]);
    }
    return hsum2(a) + hsum2(b);
}

// 8 bf16 values . x[8]
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

// the CTA's walk over blocks (<= BR rows, inside one segment) and stages
// (<= R rows of a block); identical for the producer and the consumers
struct Walk {
    uint32_t b0, b1;  // block rows [b0, b1) (virtual)
    uint32_t r0;      // first row of the current stage
    int s;            // segment
    bool ok;
};

template <int BR, class A>
__device__ __forceinline__ Walk walk_block(const A &a, uint32_t vr, uint32_t vr1)
{
    Walk w;
    w.ok = vr < vr1;
    int s = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i)
        if (i < a.nseg && vr >= a.seg[i].vbegin) s = i;
    w.s = s;
    const uint32_t send = a.seg[s].vbegin + a.seg[s].rows;
    uint32_t e = vr + BR;
    e = e < vr1 ? e : vr1;
    w.b0 = vr;
    w.b1 = e < send ? e : send;
    w.r0 = vr;
    return w;
}

template <int KIND, int MT, int P, int R>
__global__ void __launch_bounds__(kMaxCons + 32, 1) gemv_tma_kernel(const __grid_constant__ Args a)
{
    constexpr uint32_t EPV = KIND == 0 ? 16 : 8;  // values per 16-byte vector
    constexpr uint32_t ESZ = KIND == 0 ? 1 : 2;
    constexpr int BR = 32 / MT;                   // rows per reduction block
    constexpr int NST = BR / R;                   // stages per full block
    static_assert(BR % R == 0, "stage rows must divide the block");

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.stages * a.slot_bytes);
    uint64_t *empty = full + kMaxStages;
    float(*red)[32] = reinterpret_cast<float(*)[32]>(empty + kMaxStages);
    __shared__ uint32_t abort_flag;

    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t ncons = a.cons, ncw = ncons >> 5;
    const uint32_t K = a.K, S = a.stages;
    const uint32_t row_bytes = K * ESZ;
    const uint32_t vr0 = (uint32_t)(((uint64_t)blockIdx.x * a.total_rows) / gridDim.x);
    const uint32_t vr1 = (uint32_t)(((uint64_t)(blockIdx.x + 1) * a.total_rows) / gridDim.x);
    const uint32_t tok0 = blockIdx.y * MT;

    griddep_launch();
    if (t == 0) {
        for (uint32_t i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], ncw);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (t >= ncons) {
        // ---------------- producer warp: stream the rows into the ring --------
        if (lane != 0) return;
        uint32_t issued = 0;
        bool ok = true;
        for (Walk w = walk_block<BR>(a, vr0, vr1); w.ok && ok;) {
            const uint32_t slot = issued % S;
            if (issued >= S) {
                ok = mbar_wait(&empty[slot], ((issued / S) - 1) & 1);
                if (!ok || abort_flag) { abort_flag = 1; break; }
            }
            const uint32_t nrows = (w.b1 - w.r0) < (uint32_t)R ? (w.b1 - w.r0) : (uint32_t)R;
            const Seg &sg = a.seg[w.s];
            const uint32_t bytes = nrows * row_bytes;
            mbar_expect_tx(&full[slot], bytes);
            bulk_g2s(ring + (size_t)slot * a.slot_bytes, sg.W + (size_t)(w.r0 - sg.vbegin) * row_bytes, bytes,
                     &full[slot]);
            ++issued;
            w.r0 += R;
            if (w.r0 >= w.b1) w = walk_block<BR>(a, w.b1, vr1);
        }
        // wind down: every issued copy must have landed before the CTA exits
        for (uint32_t i = (issued > S ? issued - S : 0); i < issued; ++i) mbar_wait(&full[i % S], (i / S) & 1);
        return;
    }

    // ---------------- consumers --------------------------------------------
    griddep_wait();  // activations of the previous kernel are visible from here on
    float xr[P][MT][EPV];
#pragma unroll
    for (int p = 0; p < P; ++p) {
        const uint32_t k = (p * ncons + t) * EPV;
#pragma unroll
        for (int tt = 0; tt < MT; ++tt) {
            const bool v = k < K && tok0 + tt < a.m;
            const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)(tok0 + tt) * a.ldx + k);
#pragma unroll
            for (int q = 0; q < (int)EPV / 4; ++q) {
                const float4 f = v ? __ldg(xp + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                xr[p][tt][4 * q] = f.x;
                xr[p][tt][4 * q + 1] = f.y;
                xr[p][tt][4 * q + 2] = f.z;
                xr[p][tt][4 * q + 3] = f.w;
            }
        }
    }

    uint32_t consumed = 0;
    bool ok = true;
    for (Walk w = walk_block<BR>(a, vr0, vr1); w.ok && ok; w = walk_block<BR>(a, w.b1, vr1)) {
        const Seg &sg = a.seg[w.s];
        float part[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) part[i] = 0.f;
#pragma unroll
        for (int st = 0; st < NST; ++st) {
            if (ok && w.b0 + st * R < w.b1) {
                const uint32_t slot = consumed % S;
                ok = mbar_wait(&full[slot], (consumed / S) & 1);
                if (ok) {
                    const uint8_t *stage = ring + (size_t)slot * a.slot_bytes;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint32_t vr = w.b0 + st * R + r;
                        if (vr < w.b1) {
                            const uint32_t row = vr - sg.vbegin;
#pragma unroll
                            for (int p = 0; p < P; ++p) {
                                const uint32_t k = (p * ncons + t) * EPV;
                                if (k < K) {
                                    const uint4 v = *reinterpret_cast<const uint4 *>(stage + r * row_bytes + k * ESZ);
                                    if constexpr (KIND == 0) {
                                        const float sc = __ldg(sg.S + (size_t)(row >> 7) * a.kblocks + (k >> 7));
#pragma unroll
                                        for (int tt = 0; tt < MT; ++tt) {
                                            float &pr = part[(st * R + r) * MT + tt];
                                            pr = fmaf(sc, dot_fp8(v, xr[p][tt]), pr);
                                        }
                                    } else {
#pragma unroll
                                        for (int tt = 0; tt < MT; ++tt) part[(st * R + r) * MT + tt] += dot_bf16(v, xr[p][tt]);
                                    }
                                }
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                    ++consumed;
                } else {
                    abort_flag = 1;
                }
            }
        }
        if (!ok) break;
        const float v = transpose_reduce(part, lane);
        red[warp][lane] = v;
        asm volatile("bar.sync 1, %0;" ::"r"(ncons) : "memory");
        if (warp == 0) {
            float acc = red[0][lane];
            for (uint32_t q = 1; q < ncw; ++q) acc += red[q][lane];
            const uint32_t vr = w.b0 + lane / MT, tt = lane % MT;
            if (vr < w.b1 && tok0 + tt < a.m) sg.Y[(size_t)(tok0 + tt) * sg.ldy + (vr - sg.vbegin)] = acc;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(ncons) : "memory");
    }
}

// ---- FP8 decode GEMV on per-warp tensor-core MMAs ----------------------------
//
// The CUDA-core form spends ~5 issued instructions per weight byte (decode,
// widen, pack, multiply), which caps it far below HBM speed.  Here the
// multiply-accumulate runs on mma.sync.m16n8k16 (f16 x f16 -> f32):
//   A = 16 weight rows x 16 k, decoded e4m3 -> f16 by the hardware unpack
//       (exact, one instruction per two bytes, NaN codes stay NaN);
//   B = the activation, split exactly per 128-column block into
//       x * 2^e = hi + lo with hi, lo in f16 (~23 significant bits; the power
//       of two e is chosen per token and block so that max |x*2^e| < 2^15),
//       hi and lo as separate columns, up to 4 tokens per n8 MMA;
//   C = f32.  Each 128-column block's partial of a row is scaled once:
//       acc += (s[r/128, kb] * 2^-e) * C.
// Weights go straight from HBM into A fragments: lane (g, t) loads 16 bytes
// of rows g and g+8 at column 16t of a 64-column group, and byte quad j of
// that vector is its A operand for k-step j of the group (the k order inside
// the group is permuted; B is read with the same permutation from the f16
// activation columns in shared memory).  Each warp-load touches 16 rows x 64
// contiguous bytes, two full 32-byte sectors per row.  About 0.03 issued
// instructions per weight byte remain.
//
// Work: CTA c owns the contiguous rows [c*R/G, (c+1)*R/G) of the launch
// (R rows of all segments, G = grid <= SMs), cut into 16-row blocks (never
// crossing a segment).  An item is (16-row block, 256 columns = 2 blocks of
// 128); the 16 warps take items round-robin with the next item's loads in
// flight while the current one multiplies, and write one partial per item.
// After a round of row blocks, the partials of each output are added in
// column order.  Results depend only on (row, token, K): batch, multi and
// single calls agree bit for bit, and repeat exactly.
//
// K split over a cluster (standalone launches, ksplit = 2 or 4): the CTAs of
// a cluster own the same rows and each multiplies a contiguous range of the
// items' 256-column splits (and converts only that part of the activation);
// after a round, each CTA adds the partials of a share of the outputs in
// column order, reading the other CTAs' partials from their shared memory
// (distributed shared memory), so the sum is the same as without the split.
// It serves launches whose rows give each CTA a few 16-row blocks with a
// ragged last one (the 5120-row projections over 148 SMs: 34.6 rows = three
// blocks, one of 2.6 rows; a pair of CTAs holds five blocks over half the
// columns), and multi-token launches whose activation would not fit one
// CTA's shared memory otherwise.
constexpr int kM2Warps = 16;
constexpr int kM2Threads = kM2Warps * 32;
constexpr uint32_t kItemCols = 256;   // columns per work item
constexpr uint32_t kMaxRowBlocks = 256;
constexpr uint32_t kMaxChunks = 512;  // 256-column activation chunks (K <= 131072)

struct alignas(16) MArgs {
    Seg seg[4];
    const float *X;
    uint32_t K, ldx, m, kblocks, total_rows;
    uint32_t xcol_bytes;  // bytes of one f16 activation column in shared memory (2 x columns held + 32)
    uint32_t ipr;         // items per row block = ceil(K / 256)
    uint32_t rb_round;    // row blocks per round (partials buffer)
    uint32_t ksplit;      // CTAs per cluster splitting the columns (1, 2, 4)
    int nseg;
    int tp_mode;          // GemvTp::mode (m == 1 only)
    float *gathered;      // all-gather destination [world][total_rows]
    P2PView p2p;          // the ranks' exchange areas
    uint32_t *sig_count;  // HostSignal (standalone launches; null = none)
    uint32_t *sig_flag;
    uint32_t sig_seq;
};

// one 16-row block of the CTA, resolved once: weight row pointer, the
// segment's scale grid, first row in the segment, valid rows, segment
struct RowBlock {
    const uint8_t *w;
    const float *s;
    uint32_t r, nrows_seg;  // nrows_seg = valid rows | segment << 8
};

// shared-memory layout (byte offsets, 16-byte aligned)
struct MmaSmem {
    uint32_t xs, xmul, rbt, part, total;
};
__host__ __device__ __forceinline__ MmaSmem mma_smem_layout(uint32_t mt, uint32_t xcol_bytes, uint32_t kblocks,
                                                           uint32_t items_round)
{
    MmaSmem L;
    L.xs = 0;
    L.xmul = 2 * mt * xcol_bytes;
    L.rbt = (L.xmul + mt * kblocks * 4 + 15) & ~15u;
    L.part = L.rbt + kMaxRowBlocks * (uint32_t)sizeof(RowBlock);
    L.total = L.part + items_round * 16 * mt * 4;
    return L;
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint16_t f16_bits(float v)
{
    uint16_t h;
    asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(v));
    return h;
}

// Grid barrier of the chain kernel (all CTAs resident: cooperative launch),
// split in two: a CTA arrives as soon as its outputs of an op are written and
// waits only when it needs the next op's activation, after it has set up the
// next op and put its first weights in flight.  Each CTA adds one arrival per
// op boundary; boundary j is passed when the count reaches j * gridDim.x.
// Bounded; a wait that gives up records Q35CU_ERR_TIMEOUT and lets the CTA
// go on.
__device__ __forceinline__ void chain_arrive(uint32_t *bar)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(bar, 1u);
    }
}
__device__ __forceinline__ void chain_wait(uint32_t *bar, uint32_t target)
{
    if (threadIdx.x == 0) {
        uint32_t i = 0, v;
        for (;;) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if (++i >= kSpinLimit) {
                atomicExch(&g_device_status, (uint32_t)Q35CU_ERR_TIMEOUT);
                break;
            }
            if (i > 2048) __nanosleep(32);
        }
    }
    __syncthreads();
}

// One decode GEMV, run by every CTA of the grid.  The standalone kernel waits
// for the previous kernel with griddepcontrol.wait; the chain kernel (CHAIN)
// waits on its grid barrier `bar` for the previous op instead (op > 0) and
// arrives for the next one when its outputs are written (last == false).  In
// both, the warps' first two weight items are in flight when they wait.
// barrier over every thread of the cluster's CTAs (release / acquire: the
// shared-memory stores before it are visible to the other CTAs after it)
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the same shared-memory variable in the cluster's CTA r (generic address)
template <typename T>
__device__ __forceinline__ const T *cluster_peer(const T *p, uint32_t r)
{
    uint64_t out;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(p), "r"(r));
    return reinterpret_cast<const T *>(out);
}

template <int MT, bool CHAIN>
__device__ __forceinline__ void gemv_body(const MArgs &a, uint8_t *smem, const MmaSmem &L, uint32_t *xflag,
                                          uint32_t epoch, uint32_t *bar, uint32_t op, bool last = true)
{
    uint8_t *xs = smem + L.xs;                                    // [2*MT][xcol_bytes] f16 columns
    float *xmul = reinterpret_cast<float *>(smem + L.xmul);       // [MT][kblocks] 2^-e
    RowBlock *rbt = reinterpret_cast<RowBlock *>(smem + L.rbt);   // the CTA's row blocks
    float *part = reinterpret_cast<float *>(smem + L.part);       // [items in round][16 rows][MT]

    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t g = lane >> 2, tq = lane & 3;
    const uint32_t K = a.K, ipr = a.ipr, kbn = a.kblocks;
    // K split: cluster rank cr of cs takes the splits [s0, s1) of every row
    // block; the cluster's rows are those of CTA cid of ncl
    const uint32_t cs = CHAIN ? 1u : a.ksplit;
    const uint32_t cr = blockIdx.x % cs, cid = blockIdx.x / cs, ncl = gridDim.x / cs;
    const uint32_t s0 = cr * ipr / cs, s1 = (cr + 1) * ipr / cs, iw = s1 - s0;
    const uint32_t kc0 = s0 * kItemCols;  // first activation column held in shared memory
    const uint32_t vr0 = (uint32_t)(((uint64_t)cid * a.total_rows) / ncl);
    const uint32_t vr1 = (uint32_t)(((uint64_t)(cid + 1) * a.total_rows) / ncl);
    const uint32_t tok0 = blockIdx.y * MT;

    if (!CHAIN) griddep_launch();
    // the CTA's 16-row blocks, cut at segment boundaries: thread i resolves
    // block i (segment s holds ceil(len_s / 16) blocks of the CTA's rows)
    uint32_t nrb = 0;
    for (int s = 0; s < a.nseg; ++s) {
        const Seg &sg = a.seg[s];
        const uint32_t lo = vr0 > sg.vbegin ? vr0 : sg.vbegin, e = sg.vbegin + sg.rows;
        const uint32_t hi = vr1 < e ? vr1 : e;
        const uint32_t nb = hi > lo ? (hi - lo + 15) / 16 : 0;
        if (t >= nrb && t < nrb + nb && t < kMaxRowBlocks) {
            const uint32_t vr = lo + (t - nrb) * 16, ve = vr + 16 < hi ? vr + 16 : hi;
            RowBlock rb;
            rb.r = vr - sg.vbegin;
            rb.w = sg.W + (size_t)rb.r * K;
            rb.s = sg.S;
            rb.nrows_seg = (ve - vr) | ((uint32_t)s << 8);
            rbt[t] = rb;
        }
        nrb += nb;
    }
    nrb = nrb < kMaxRowBlocks ? nrb : kMaxRowBlocks;
    __syncthreads();

    // this lane's loads of an item: rows g, g+8 x 4 groups of 64 columns, and
    // the block scales of both rows.  Out-of-range rows and columns read a
    // clamped in-range address instead of being predicated off: their
    // products land only in rows / blocks that are never stored.
    auto issue = [&](uint4 (&v)[8], float (&sc)[4], uint32_t rbi, uint32_t sp) {
        const RowBlock rb = rbt[rbi];
        const uint32_t nrows = rb.nrows_seg & 0xFF, c0 = sp * kItemCols;
        const uint32_t g0 = g < nrows ? g : nrows - 1, g1 = g + 8 < nrows ? g + 8 : nrows - 1;
        const uint8_t *w0 = rb.w + (size_t)g0 * K + c0 + tq * 16;
        const uint8_t *w1 = rb.w + (size_t)g1 * K + c0 + tq * 16;
        const uint32_t c1 = c0 + 128 < K ? 128u : 0u;  // second block of the item (re-read if past K)
        v[0] = ld_stream(w0);
        v[1] = ld_stream(w1);
        v[2] = ld_stream(w0 + 64);
        v[3] = ld_stream(w1 + 64);
        v[4] = ld_stream(w0 + c1);
        v[5] = ld_stream(w1 + c1);
        v[6] = ld_stream(w0 + c1 + 64);
        v[7] = ld_stream(w1 + c1 + 64);
        const float *s0 = rb.s + (size_t)((rb.r + g0) >> 7) * kbn + (c0 >> 7);
        const float *s1 = rb.s + (size_t)((rb.r + g1) >> 7) * kbn + (c0 >> 7);
        const uint32_t d1 = c1 >> 7;
        sc[0] = __ldg(s0);
        sc[1] = __ldg(s1);
        sc[2] = __ldg(s0 + d1);
        sc[3] = __ldg(s1 + d1);
    };

    // multiply one item (2 blocks of 128 columns) held in v; write its partial.
    // Lanes with g >= 2*MT feed B columns no output reads: they load a live
    // column (finite data) rather than zeros, as MMA output columns never mix.
    // (biased by the first column held, kc0: indexed with absolute columns)
    const uint8_t *xcol = xs + (size_t)(g % (2 * MT)) * a.xcol_bytes + tq * 32 - (size_t)kc0 * 2;
    auto compute = [&](const uint4 (&v)[8], const float (&sc)[4], uint32_t sp, uint32_t slot) {
        const uint32_t c0 = sp * kItemCols;
        if (MT == 1 && !CHAIN) {  // this item's activation chunk is converted (bounded wait)
            if (lane == 0) {
                for (uint32_t i = 0; *reinterpret_cast<volatile uint32_t *>(&xflag[sp]) != epoch; ++i)
                    if (i >= kSpinLimit) {
                        atomicExch(&g_device_status, (uint32_t)Q35CU_ERR_TIMEOUT);
                        break;
                    }
                __threadfence_block();
            }
            __syncwarp();
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
            const uint32_t kb = (c0 >> 7) + hb;
            if (kb < kbn) {
                float cz[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint4 A0 = v[2 * (2 * hb + q)], A1 = v[2 * (2 * hb + q) + 1];
                    const uint32_t w0[4] = {A0.x, A0.y, A0.z, A0.w}, w1[4] = {A1.x, A1.y, A1.z, A1.w};
                    const uint8_t *xb = xcol + (size_t)(c0 + hb * 128 + q * 64) * 2;
                    const uint4 b01 = *reinterpret_cast<const uint4 *>(xb);
                    const uint4 b23 = *reinterpret_cast<const uint4 *>(xb + 16);
                    const uint32_t bw[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t a0, a2, a1, a3;
                        hw_f16x2(w0[j], a0, a2);
                        hw_f16x2(w1[j], a1, a3);
                        mma16816(cz, a0, a1, a2, a3, bw[2 * j], bw[2 * j + 1]);
                    }
                }
                const float xm = xmul[(tq < MT ? tq : 0) * kbn + kb];
                const float f0 = sc[2 * hb] * xm, f1 = sc[2 * hb + 1] * xm;
                acc[0] = fmaf(f0, cz[0], acc[0]);
                acc[1] = fmaf(f0, cz[1], acc[1]);
                acc[2] = fmaf(f1, cz[2], acc[2]);
                acc[3] = fmaf(f1, cz[3], acc[3]);
            }
        }
        // lane (g, tq) holds token tq of rows g and g+8 as (hi, lo) column pairs
        if (tq < MT) {
            part[((size_t)slot * 16 + g) * MT + tq] = acc[0] + acc[1];
            part[((size_t)slot * 16 + g + 8) * MT + tq] = acc[2] + acc[3];
        }
    };

    // items of this warp in round order: (row block, split in [s0, s1))
    // advanced by 16 items
    const uint32_t nitems = nrb * iw;
    uint32_t it = warp, rbi = warp / iw, sp = s0 + warp % iw;
    auto advance = [&]() {
        it += kM2Warps;
        sp += kM2Warps;
        while (sp >= s1) { sp -= iw; ++rbi; }
    };

    // issue cursor (items are issued in compute order, two ahead of the one
    // being multiplied)
    uint32_t jt = it, rbj = rbi, sj = sp;
    auto advance_issue = [&]() {
        jt += kM2Warps;
        sj += kM2Warps;
        while (sj >= s1) { sj -= iw; ++rbj; }
    };
    uint4 va[8], vb[8];
    float sa[4], sb[4];
    // weights only: the warp's first two items are in flight before it waits
    // for the previous kernel (or op)
    if (jt < nitems) { issue(va, sa, rbj, sj); advance_issue(); }
    if (jt < nitems) { issue(vb, sb, rbj, sj); advance_issue(); }
    if (!CHAIN)
        griddep_wait();
    else if (op > 0)
        chain_wait(bar, op * gridDim.x);
    // activation -> f16 hi/lo columns, one 128-column block at a time
    auto convert_block = [&](uint32_t tt, uint32_t kb, const float4 &v) {
        const uint32_t k = kb * 128 + lane * 4;
        float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        int e = 0;  // 2^e with max |x*2^e| < 2^15; |e| <= 126 keeps 2^e and 2^-e normal
        if (mx > 0.f && mx <= 3.402823466e38f) {
            const int E = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;
            e = 14 - E;
            e = e > 126 ? 126 : (e < -126 ? -126 : e);
        }
        const float up = __uint_as_float((uint32_t)(e + 127) << 23);
        const float down = __uint_as_float((uint32_t)(127 - e) << 23);
        const float xv[4] = {v.x * up, v.y * up, v.z * up, v.w * up};
        uint16_t hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            hi[j] = f16_bits(xv[j]);
            lo[j] = f16_bits(xv[j] - __half2float(__ushort_as_half(hi[j])));
        }
        *reinterpret_cast<uint2 *>(xs + (size_t)(2 * tt) * a.xcol_bytes + (k - kc0) * 2) =
            make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
        *reinterpret_cast<uint2 *>(xs + (size_t)(2 * tt + 1) * a.xcol_bytes + (k - kc0) * 2) =
            make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
        if (lane == 0) xmul[tt * kbn + kb] = down;
    };
    // chunk flags in standalone launches (the chain converts with a barrier:
    // its kernel has no registers to spare for the flag bookkeeping)
    constexpr bool FLAGS = MT == 1 && !CHAIN;
    if (FLAGS) {
        // Warp w converts the column chunks w, w + 16, ... (a chunk = the two
        // blocks of one item; its own first item's chunk comes first) and
        // marks each chunk ready with this op's epoch: a warp then waits only
        // for the chunks of the item it multiplies, not for the whole vector.
        // (this CTA's chunks: the splits [s0, s1))
        const uint32_t nchunk = s1;
        for (uint32_t c0 = s0 + warp; c0 < nchunk; c0 += 4 * kM2Warps) {
            float4 xv4[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t c = c0 + (u >> 1) * kM2Warps, kb = 2 * c + (u & 1);
                xv4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (c < nchunk && kb < kbn && tok0 < a.m)
                    xv4[u] = __ldcg(reinterpret_cast<const float4 *>(a.X + (size_t)tok0 * a.ldx + kb * 128 + lane * 4));
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t c = c0 + (u >> 1) * kM2Warps, kb = 2 * c + (u & 1);
                if (c >= nchunk) break;
                if (kb < kbn) convert_block(0, kb, xv4[u]);
                if (u & 1) {
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        *reinterpret_cast<volatile uint32_t *>(&xflag[c]) = epoch;
                    }
                }
            }
        }
    } else {
        // one warp per (token, 128-column block), XU blocks of a warp loaded
        // at once so their L2 round trips overlap
        // (this CTA's blocks: [2 s0, min(2 s1, kblocks)))
        constexpr int XU = MT == 1 ? 8 : 4;
        const uint32_t kb0 = 2 * s0, kbl = (2 * s1 < kbn ? 2 * s1 : kbn) - kb0;
        for (uint32_t base = warp; base < MT * kbl; base += XU * kM2Warps) {
            float4 xv4[XU];
#pragma unroll
            for (int u = 0; u < XU; ++u) {
                const uint32_t idx = base + u * kM2Warps;
                const uint32_t tt = idx / kbl, kb = kb0 + idx % kbl;
                xv4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (idx < MT * kbl && tok0 + tt < a.m)
                    xv4[u] = __ldcg(reinterpret_cast<const float4 *>(a.X + (size_t)(tok0 + tt) * a.ldx + kb * 128 + lane * 4));
            }
#pragma unroll
            for (int u = 0; u < XU; ++u) {
                const uint32_t idx = base + u * kM2Warps;
                if (idx >= MT * kbl) break;
                convert_block(idx / kbl, kb0 + idx % kbl, xv4[u]);
            }
        }
    }
    __shared__ uint32_t tp_seq_s;
    if (MT == 1 && a.tp_mode && t == 0) tp_seq_s = p2p_next_seq(a.p2p);  // the previous kernel has completed
    if (!FLAGS) __syncthreads();  // the whole activation is converted

    bool flip = false;  // the warp's next item sits in vb
    for (uint32_t rb0 = 0; rb0 < nrb; rb0 += a.rb_round) {
        const uint32_t nrb_r = (nrb - rb0) < a.rb_round ? (nrb - rb0) : a.rb_round;
        const uint32_t iend = (rb0 + nrb_r) * iw;  // items of this round: [rb0 * iw, iend)
        // ping-pong: buffer P holds item it, Q the next one; a buffer is
        // refilled with the item two ahead as soon as it has been multiplied.
        // Returns true when the round ends with the next item in Q.
        auto run = [&](uint4 (&P)[8], float (&Ps)[4], uint4 (&Q)[8], float (&Qs)[4]) -> bool {
            while (it < iend) {
                compute(P, Ps, sp, it - rb0 * iw);
                advance();
                if (jt < nitems) { issue(P, Ps, rbj, sj); advance_issue(); }
                if (it >= iend) return true;
                compute(Q, Qs, sp, it - rb0 * iw);
                advance();
                if (jt < nitems) { issue(Q, Qs, rbj, sj); advance_issue(); }
            }
            return false;
        };
        flip ^= flip ? run(vb, sb, va, sa) : run(va, sa, vb, sb);
        __syncthreads();
        if (cs > 1) cluster_sync_all();  // every CTA of the cluster has its partials
        // combine: output (row i of block, token tt) = sum over the block's
        // items, in column order (under a K split: outputs cr, cr + cs, ...
        // of the round, the splits of CTA r read from its shared memory)
        for (uint32_t o = t * cs + cr; o < nrb_r * 16 * MT; o += kM2Threads * cs) {
            const uint32_t rbl = o / (16 * MT), i = (o / MT) % 16, tt = o % MT;
            const RowBlock rb = rbt[rb0 + rbl];
            if (i >= (rb.nrows_seg & 0xFF) || tok0 + tt >= a.m) continue;
            // the partials are loaded 8 at a time and added in column order:
            // the loads' round trips (distributed shared memory under a K
            // split) overlap, the sum is the same
            float y = 0.f;
            auto sum_splits = [&](const float *pp, uint32_t n) {
                uint32_t s = 0;
                for (; s + 8 <= n; s += 8) {
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = pp[(size_t)(s + u) * 16 * MT];
#pragma unroll
                    for (int u = 0; u < 8; ++u) y += v[u];
                }
                for (; s < n; ++s) y += pp[(size_t)s * 16 * MT];
            };
            if (cs == 1) {
                sum_splits(part + ((size_t)(rbl * ipr) * 16 + i) * MT + tt, ipr);
            } else {
                for (uint32_t r = 0; r < cs; ++r) {
                    const uint32_t r0 = r * ipr / cs, rw = (r + 1) * ipr / cs - r0;
                    sum_splits(cluster_peer(part, r) + ((size_t)(rbl * rw) * 16 + i) * MT + tt, rw);
                }
            }
            const Seg &sg = a.seg[rb.nrows_seg >> 8];
            if (MT == 1 && a.tp_mode) {  // one token: publish the row to every rank
                const uint32_t v = sg.vbegin + rb.r + i, tp_seq = tp_seq_s;
                for (int d = 0; d < a.p2p.world; ++d) p2p_put(p2p_slot(a.p2p.area[d], tp_seq, a.p2p.rank) + v, y, tp_seq);
                if (a.tp_mode == 1) continue;  // all-reduce: Y is the cross-rank sum, written below
            }
            sg.Y[(size_t)(tok0 + tt) * sg.ldy + rb.r + i] = y;
        }
        if (cs > 1)
            cluster_sync_all();  // the partials were read: the next round may overwrite them, or the CTA leave
        else
            __syncthreads();
    }

    // Tensor-parallel epilogue (one token).  Every rank splits the rows over
    // CTAs the same way, so this CTA only needs its peers' words for its own
    // rows [vr0, vr1): no grid-wide barrier, no separate collective kernel.
    if (MT == 1 && a.tp_mode) {
        uint8_t *mine = a.p2p.area[a.p2p.rank];
        const uint32_t tp_seq = tp_seq_s;
        for (uint32_t v = vr0 + t; v < vr1; v += kM2Threads) {
            if (a.tp_mode == 1) {
                float y = 0.f;
                for (int q = 0; q < a.p2p.world; ++q) y += p2p_get(p2p_slot(mine, tp_seq, q) + v, tp_seq, &g_device_status);
                int s = 0;
                for (int j = 1; j < a.nseg; ++j)
                    if (v >= a.seg[j].vbegin) s = j;
                a.seg[s].Y[v - a.seg[s].vbegin] = y;
            } else {
                for (int q = 0; q < a.p2p.world; ++q)
                    a.gathered[(size_t)q * a.total_rows + v] = p2p_get(p2p_slot(mine, tp_seq, q) + v, tp_seq, &g_device_status);
            }
        }
        __syncthreads();
        if (t == 0) p2p_finish(a.p2p, tp_seq);
    }
    if (CHAIN && !last) chain_arrive(bar);
}

template <int MT>
__global__ void __launch_bounds__(kM2Threads, 1) gemv_mma_kernel(const __grid_constant__ MArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint32_t xflag[kMaxChunks];
    for (uint32_t i = threadIdx.x; i < kMaxChunks; i += kM2Threads) xflag[i] = 0;  // ordered by the body's first barrier
    const MmaSmem L = mma_smem_layout(MT, a.xcol_bytes, a.kblocks, a.rb_round * ((a.ipr + a.ksplit - 1) / a.ksplit));
    gemv_body<MT, false>(a, smem, L, xflag, 1, nullptr, 0);
    if (a.sig_flag) {
        // host-pointer call: the last CTA out tells the waiting host thread,
        // through host-mapped memory, that every output is visible
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence_system();  // this CTA's outputs (host-mapped) before its count
            const uint32_t ctas = gridDim.x * gridDim.y;
            if (atomicAdd(a.sig_count, 1u) == ctas - 1) {
                __threadfence_system();
                *a.sig_count = 0;
                volatile uint32_t *f = a.sig_flag;
                f[1] = *reinterpret_cast<volatile uint32_t *>(&g_device_status);
                __threadfence_system();
                f[0] = a.sig_seq;
            }
        }
    }
}


// A chain of one-token decode GEMVs in one cooperative launch: every CTA
// walks the ops in order with a grid barrier before each op after the first,
// so no launch ramp or tail separates two projections and each op's first
// weights are in flight before the barrier.  The op descriptors live in
// device memory; the shared-memory layout is the largest op's.
struct ChainArgs {
    const MArgs *ops;
    uint32_t nops;
    uint32_t *bar;     // [0] barrier count, [1] exit ticket; zero at launch, reset at exit
    MmaSmem L;
};

__global__ void __launch_bounds__(kM2Threads, 1) gemv_chain_kernel(const __grid_constant__ ChainArgs c)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ MArgs op_s[2];
    constexpr uint32_t kOpVecs = sizeof(MArgs) / 16;
    static_assert(sizeof(MArgs) % 16 == 0, "op descriptors move in 16-byte pieces");
    // the descriptors travel through L2 into shared memory one op ahead
    auto fetch_op = [&](uint32_t k) {
        if (threadIdx.x < kOpVecs)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(reinterpret_cast<uint4 *>(&op_s[k & 1]) + threadIdx.x)),
                         "l"(reinterpret_cast<const uint4 *>(c.ops + k) + threadIdx.x)
                         : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch_op(0);
    for (uint32_t k = 0; k < c.nops; ++k) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();  // op k's descriptor has landed; the previous op is done with the other one and shared memory
        if (k + 1 < c.nops) fetch_op(k + 1);
        gemv_body<1, true>(op_s[k & 1], smem, c.L, nullptr, 0, c.bar, k, k + 1 == c.nops);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // the last CTA out resets the counters for the next launch
        __threadfence();
        if (atomicAdd(c.bar + 1, 1u) == gridDim.x - 1) {
            c.bar[0] = 0;
            c.bar[1] = 0;
            __threadfence();
        }
    }
}

// Any shape, any alignment: one warp per (row, token), lanes over k, one
// value per lane per step.  Used only when cols is not a multiple of the
// 16-byte vector, an activation row is not 16-byte aligned, or K needs more
// register passes than the streaming kernel keeps (the odd shapes of the
// reference's known-answer tests, e.g. 3x5 and 129x129).
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

__device__ __forceinline__ bool nan_code(uint32_t w) { return __vcmpeq4(w | 0x80808080u, 0xFFFFFFFFu) != 0u; }

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
int launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const Args &a)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
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

template <int KIND, int MT, int P, int R>
int launch_tma(const Args &a, dim3 grid, size_t smem, cudaStream_t st)
{
    auto k = gemv_tma_kernel<KIND, MT, P, R>;
    static bool configured[64] = {};  // per instantiation and device
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 224 * 1024));
        configured[dev] = true;
    }
    return launch_pdl(k, grid, dim3(a.cons + 32), smem, st, a);
}

constexpr uint32_t kMmaSmemAttr = 220 * 1024;

template <int MT>
int mma_configure(int dev)
{
    static bool configured[64] = {};
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(gemv_mma_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMmaSmemAttr));
        configured[dev] = true;
    }
    return Q35CU_OK;
}

template <int MT>
int launch_mma(const MArgs &a, dim3 grid, size_t smem, cudaStream_t st)
{
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    int rc = mma_configure<MT>(dev);
    if (rc) return rc;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kM2Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.ksplit;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.ksplit > 1 ? 2 : 1;
    Q35CU_CUDA(cudaLaunchKernelEx(&cfg, gemv_mma_kernel<MT>, a));
    count_launch();
    return Q35CU_OK;
}

// clusters of cs CTAs of gemv_mma_kernel<MT> that the device holds at once
// (one CTA per SM; cached per device)
template <int MT>
uint32_t mma_max_clusters(uint32_t cs)
{
    static int cache[64][5] = {};  // [device][cs]: 0 = not asked, -1 = none
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || cs > 4) return 0;
    int &c = cache[dev][cs];
    if (c == 0) {
        c = -1;
        if (mma_configure<MT>(dev) == Q35CU_OK) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(cs * 64);
            cfg.blockDim = dim3(kM2Threads);
            cfg.dynamicSmemBytes = kMmaSmemAttr - 4096;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = cs;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, gemv_mma_kernel<MT>, &cfg) == cudaSuccess && n > 0) c = n;
            cudaGetLastError();  // an unsupported query leaves no error behind
        }
    }
    return c > 0 ? (uint32_t)c : 0u;
}

// FP8 weights with cols % 128 == 0: the tensor-core decode GEMV
int launch_gemv_mma(const Args &a0, cudaStream_t st, const GemvTp &tp, const HostSignal *sig)
{
    MArgs a{};
    if (sig) {
        a.sig_count = sig->count;
        a.sig_flag = sig->flag;
        a.sig_seq = sig->seq;
    }
    for (int s = 0; s < 4; ++s) a.seg[s] = a0.seg[s];
    a.X = a0.X;
    a.K = a0.K;
    a.ldx = a0.ldx;
    a.m = a0.m;
    a.kblocks = a0.kblocks;
    a.total_rows = a0.total_rows;
    a.nseg = a0.nseg;
    a.ipr = (a0.K + kItemCols - 1) / kItemCols;
    a.tp_mode = tp.mode;
    a.gathered = tp.gathered;
    if (tp.mode) {
        if (a0.m != 1) return set_error(Q35CU_ERR_UNSUPPORTED, "gemv: the tensor-parallel epilogue takes one token");
        if (!p2p_view(&a.p2p)) return set_error(Q35CU_ERR_NCCL, "gemv: p2p collectives not open");
        if (a0.total_rows > kP2PMaxElems) return set_error(Q35CU_ERR_UNSUPPORTED, "gemv: %u rows exceed the exchange area", a0.total_rows);
        if (tp.mode == 2 && !tp.gathered) return set_error(Q35CU_ERR_ARG, "gemv: all-gather needs a destination");
    }
    const uint32_t budget = 216 * 1024;
    const uint32_t sms = (uint32_t)device_sms();
    const uint32_t gx1 = ((a.total_rows + 15) / 16) < sms ? (a.total_rows + 15) / 16 : sms;
    if ((a.kblocks + 1) / 2 > kMaxChunks) return set_error(Q35CU_ERR_UNSUPPORTED, "gemv: cols %u too large", a0.K);
    const int mt_want = a0.m >= 3 ? 4 : (int)a0.m;
    // One geometry per column split cs (CTAs per cluster): grid, row blocks
    // of the busiest CTA, token tile and shared-memory layout.  Cost = the
    // items (16-row block x 256 columns) the busiest CTA multiplies times the
    // token tiles each row range is streamed for, plus kSplitCost items for
    // the cluster's hand-off; the cheapest wins (Q35CU_GEMV_KSPLIT = 1, 2 or
    // 4 forces one).  Tensor-parallel launches keep cs = 1: their epilogue
    // exchanges each CTA's own rows.
    struct Geo {
        uint32_t cs, gx, nrb_max, iw, xcol, mt, rbr, gy;
        size_t smem;
        uint64_t cost;
    };
    uint32_t split_cost = 16;
    if (const char *e = getenv("Q35CU_GEMV_KSPLIT_COST")) split_cost = (uint32_t)strtoul(e, nullptr, 10);
    int forced = 0;
    if (const char *e = getenv("Q35CU_GEMV_KSPLIT")) forced = atoi(e);
    auto geometry = [&](uint32_t cs, Geo &g) -> bool {
        g.cs = cs;
        g.gx = gx1 / cs * cs;
        if (!g.gx || (cs > 1 && (tp.mode || a.ipr < cs))) return false;
        if (cs > 1) {
            // as many clusters as the device holds at once (clusters of 4
            // do not tile every GPC: fewer than SMs / 4 of them fit)
            const uint32_t ncl_max = mma_max_clusters<1>(cs);
            if (!ncl_max) return false;
            if (ncl_max < g.gx / cs) g.gx = ncl_max * cs;
        }
        const uint32_t rows_cl = (a.total_rows + g.gx / cs - 1) / (g.gx / cs);
        g.nrb_max = (rows_cl + 15) / 16 + 2 * (uint32_t)a.nseg;
        if (g.nrb_max > kMaxRowBlocks) return false;
        g.iw = (a.ipr + cs - 1) / cs;
        const uint32_t kloc = g.iw * kItemCols < a0.K ? g.iw * kItemCols : a0.K;
        g.xcol = 2 * kloc + 32;
        auto fits = [&](int mtt, uint32_t rbr) {
            return mma_smem_layout(mtt, g.xcol, a.kblocks, rbr * g.iw).total <= budget;
        };
        int mt = mt_want;
        while (mt > 1 && !fits(mt, 1)) mt /= 2;
        if (!fits(mt, 1)) return false;
        // row blocks per round: all of the CTA's if they fit, else as many as fit
        uint32_t rbr = g.nrb_max;
        while (rbr > 1 && !fits(mt, rbr)) --rbr;
        g.mt = (uint32_t)mt;
        g.rbr = rbr;
        g.smem = mma_smem_layout(mt, g.xcol, a.kblocks, rbr * g.iw).total;
        g.gy = (a0.m + mt - 1) / mt;
        const uint32_t blocks = (rows_cl + 15) / 16 + (uint32_t)a.nseg - 1;
        g.cost = (uint64_t)blocks * g.iw * g.gy + (cs > 1 ? split_cost : 0);
        return true;
    };
    // Shared memory above kSmemSoft is taken from the L1 that holds the
    // weight loads in flight: a geometry within it wins over any beyond it
    // (5120x17408 at 4 tokens: 4-CTA split, 122 KB, 33.4 us against the
    // 2-CTA split, 207 KB, 42.8 us, at equal item cost).
    constexpr size_t kSmemSoft = 160 * 1024;
    Geo best{}, cand{};
    bool have = false;
    for (uint32_t cs : {1u, 2u, 4u}) {
        if (forced && (uint32_t)forced != cs) continue;
        if (!geometry(cs, cand)) continue;
        const bool soft = cand.smem <= kSmemSoft, best_soft = have && best.smem <= kSmemSoft;
        if (!have || (soft && !best_soft) || (soft == best_soft && cand.cost < best.cost)) {
            best = cand;
            have = true;
        }
    }
    if (!have && forced) have = geometry(1, best);
    if (!have) return set_error(Q35CU_ERR_UNSUPPORTED, "gemv: %u rows x %u cols do not fit a CTA", a.total_rows, a0.K);
    a.ksplit = best.cs;
    a.xcol_bytes = best.xcol;
    a.rb_round = best.rbr;
    const int mt = (int)best.mt;
    const uint32_t gx = best.gx;
    const size_t smem = best.smem;
    const uint32_t gy = best.gy;
    if (gy > 65535) return set_error(Q35CU_ERR_ARG, "gemv: too many tokens (%u)", a0.m);
    const dim3 grid(gx, gy);
    if (mt == 1) return launch_mma<1>(a, grid, smem, st);
    if (mt == 2) return launch_mma<2>(a, grid, smem, st);
    return launch_mma<4>(a, grid, smem, st);
}

// (MT, P) with MT * P <= 4 registers of activation per thread-slice; R rows
// per stage from P.  A bulk copy costs about the same per instruction at any
// size, so stages are as large as the ring allows: the lm_head's 5120-column
// bf16 rows (P = 2) go 8 rows = 80 KB per copy, two stages (6.6 TB/s against
// 5.1 at 2 rows and five stages, 6.0 at 4 rows; same bits).
template <int KIND>
int dispatch_tma(const Args &a, dim3 grid, size_t smem, int mt, int P, cudaStream_t st)
{
    if (P == 1) {
        if (mt == 1) return launch_tma<KIND, 1, 1, 4>(a, grid, smem, st);
        if (mt == 2) return launch_tma<KIND, 2, 1, 4>(a, grid, smem, st);
        return launch_tma<KIND, 4, 1, 4>(a, grid, smem, st);
    }
    if (P == 2) {
        if (mt == 1) return launch_tma<KIND, 1, 2, 8>(a, grid, smem, st);
        return launch_tma<KIND, 2, 2, 8>(a, grid, smem, st);
    }
    if (P == 3) return launch_tma<KIND, 1, 3, 1>(a, grid, smem, st);
    return launch_tma<KIND, 1, 4, 1>(a, grid, smem, st);
}

}  // namespace

// consumer threads and passes of the streaming kernel: a function of K only
void gemv_geometry(int kind, uint32_t K, uint32_t *threads, uint32_t *passes)
{
    const uint32_t epv = kind == 0 ? 16 : 8;
    const uint32_t nvec = (K + epv - 1) / epv;
    const uint32_t P = (nvec + kMaxCons - 1) / kMaxCons;
    uint32_t T = (nvec + P - 1) / P;
    T = (T + 31) / 32 * 32;
    *threads = T;
    *passes = P;
}

// ---- the decode chain (host side) -----------------------------------------
size_t chain_op_bytes() { return sizeof(MArgs); }

// one op of a chain: the launch arguments of launch_gemv_mma for one token,
// with the grid fixed at one CTA per SM (rb_round is set by chain_layout)
int chain_build_op(const GemvSeg *segs_in, int nseg, const float *X, uint32_t K, const GemvTp &tp, void *out)
{
    if (nseg < 1 || nseg > 4 || !X || K == 0) return set_error(Q35CU_ERR_ARG, "chain: bad op");
    if (K % 128 || (uintptr_t)X % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "chain: cols %u (needs a multiple of 128)", K);
    MArgs a{};
    uint32_t vb = 0;
    for (int s = 0; s < nseg; ++s) {
        const GemvSeg &g = segs_in[s];
        if ((uintptr_t)g.W % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "chain: misaligned weight");
        a.seg[s] = Seg{g.W, g.S, g.Y, g.rows, g.ldy, vb, g.has_nan};
        vb += g.rows;
    }
    a.X = X;
    a.K = K;
    a.ldx = K;
    a.m = 1;
    a.kblocks = K / 128;
    a.total_rows = vb;
    a.nseg = nseg;
    a.xcol_bytes = 2 * K + 32;
    a.ipr = (K + kItemCols - 1) / kItemCols;
    a.tp_mode = tp.mode;
    a.gathered = tp.gathered;
    if (tp.mode) {
        if (!p2p_view(&a.p2p)) return set_error(Q35CU_ERR_NCCL, "chain: p2p collectives not open");
        if (vb > kP2PMaxElems) return set_error(Q35CU_ERR_UNSUPPORTED, "chain: %u rows exceed the exchange area", vb);
        if (tp.mode == 2 && !tp.gathered) return set_error(Q35CU_ERR_ARG, "chain: all-gather needs a destination");
    }
    const uint32_t sms = (uint32_t)device_sms();
    const uint32_t rows_cta = (vb + sms - 1) / sms;
    if ((rows_cta + 15) / 16 + 2 * (uint32_t)nseg > kMaxRowBlocks) return set_error(Q35CU_ERR_UNSUPPORTED, "chain: rows");
    memcpy(out, &a, sizeof(a));
    return Q35CU_OK;
}

// the shared-memory layout every op of the chain fits in; sets each op's
// rows-per-round.  layout_out: {xs, xmul, rbt, part, total} bytes.
int chain_layout(void *ops, uint32_t nops, uint32_t layout_out[5])
{
    MArgs *o = static_cast<MArgs *>(ops);
    uint32_t xcol = 0, kb = 0, ipr_max = 0;
    for (uint32_t i = 0; i < nops; ++i) {
        xcol = o[i].xcol_bytes > xcol ? o[i].xcol_bytes : xcol;
        kb = o[i].kblocks > kb ? o[i].kblocks : kb;
        ipr_max = o[i].ipr > ipr_max ? o[i].ipr : ipr_max;
    }
    // Shared memory is sized to what the ops need, not to the budget: every
    // byte above that is taken from L1, which holds the weight loads in flight.
    const uint32_t budget = 216 * 1024;
    MmaSmem L = mma_smem_layout(1, xcol, kb, 0);
    if (L.part + ipr_max * 16 * 4 > budget) return set_error(Q35CU_ERR_UNSUPPORTED, "chain: cols too large");
    const uint32_t sms = (uint32_t)device_sms();
    uint32_t need = 0;  // partial slots for every op to run in one round
    for (uint32_t i = 0; i < nops; ++i) {
        const uint32_t rows_cta = (o[i].total_rows + sms - 1) / sms;
        const uint32_t nrb_max = (rows_cta + 15) / 16 + 2 * (uint32_t)o[i].nseg;
        need = nrb_max * o[i].ipr > need ? nrb_max * o[i].ipr : need;
    }
    const uint32_t cap = (budget - L.part) / (16 * 4);
    const uint32_t slots = need < cap ? need : cap;
    for (uint32_t i = 0; i < nops; ++i) {
        const uint32_t rows_cta = (o[i].total_rows + sms - 1) / sms;
        const uint32_t nrb_max = (rows_cta + 15) / 16 + 2 * (uint32_t)o[i].nseg;
        uint32_t rbr = slots / o[i].ipr;
        rbr = rbr < 1 ? 1 : (rbr > nrb_max ? nrb_max : rbr);
        o[i].rb_round = rbr;
    }
    L.total = L.part + slots * 16 * 4;
    layout_out[0] = L.xs;
    layout_out[1] = L.xmul;
    layout_out[2] = L.rbt;
    layout_out[3] = L.part;
    layout_out[4] = L.total;
    return Q35CU_OK;
}

int launch_chain(const void *d_ops, uint32_t nops, uint32_t *d_bar, const uint32_t layout[5], cudaStream_t st)
{
    if (!nops) return Q35CU_OK;
    static bool configured[64] = {};
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        configured[dev] = true;
    }
    ChainArgs c{};
    c.ops = static_cast<const MArgs *>(d_ops);
    c.nops = nops;
    c.bar = d_bar;
    c.L = MmaSmem{layout[0], layout[1], layout[2], layout[3], layout[4]};
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)device_sms());
    cfg.blockDim = dim3(kM2Threads);
    cfg.dynamicSmemBytes = layout[4];
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barrier cannot wait on an unscheduled CTA
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35CU_CUDA(cudaLaunchKernelEx(&cfg, gemv_chain_kernel, c));
    count_launch();
    return Q35CU_OK;
}

int launch_gemv(int kind, const GemvSeg *segs_in, int nseg, const float *X, uint32_t K, uint32_t ldx, uint32_t m,
                cudaStream_t st, const GemvTp &tp, const HostSignal *sig)
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
    const uint32_t esz = kind == 0 ? 1 : 2;
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
    if (vec_ok && kind == 0 && K % 128 == 0 && getenv("Q35CU_GEMV_SIMT") == nullptr) return launch_gemv_mma(a, st, tp, sig);
    if (tp.mode) return set_error(Q35CU_ERR_UNSUPPORTED, "gemv: the tensor-parallel epilogue needs the tensor-core GEMV");
    if (sig) return set_error(Q35CU_ERR_UNSUPPORTED, "gemv: the completion signal needs the tensor-core GEMV");
    uint32_t T = 0, P = 0;
    gemv_geometry(kind, K, &T, &P);
    if (P > 4) vec_ok = false;
    if (vec_ok) {
        a.cons = T;
        const int R = P == 1 ? 4 : (P == 2 ? 8 : 1);
        a.slot_bytes = (uint32_t)R * K * esz;
        uint32_t stages = kRingBudget / a.slot_bytes;
        stages = stages < 2 ? 2 : (stages > kMaxStages ? kMaxStages : stages);
        a.stages = stages;
        const size_t smem = (size_t)stages * a.slot_bytes + 2 * kMaxStages * 8 + kMaxWarps * 32 * 4;
        const int mt_max = (int)(4 / P);
        int mt = m == 1 ? 1 : (m == 2 ? 2 : 4);
        if (mt > mt_max) mt = mt_max;
        const uint32_t sms = (uint32_t)device_sms();
        const uint32_t gx = vb < sms ? vb : sms;
        const uint32_t gy = (m + mt - 1) / mt;
        if (gy > 65535) return set_error(Q35CU_ERR_ARG, "gemv: too many tokens (%u)", m);
        const dim3 grid(gx, gy);
        return kind == 0 ? dispatch_tma<0>(a, grid, smem, mt, (int)P, st)
                         : dispatch_tma<1>(a, grid, smem, mt, (int)P, st);
    }
    const uint64_t items = (uint64_t)vb * m;
    const uint64_t blocks = (items + 7) / 8;
    if (blocks > 0x7FFFFFFFull) return set_error(Q35CU_ERR_ARG, "gemv: shape too large for the generic kernel");
    if (kind == 0) return launch_pdl(gemv_any_kernel<0>, dim3((unsigned)blocks), dim3(256), 0, st, a);
    return launch_pdl(gemv_any_kernel<1>, dim3((unsigned)blocks), dim3(256), 0, st, a);
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

uint32_t *device_status_word()
{
    void *p = nullptr;
    return cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess ? static_cast<uint32_t *>(p) : nullptr;
}

int device_status(uint32_t *status, bool clear)
{
    Q35CU_CUDA(cudaMemcpyFromSymbol(status, g_device_status, 4));
    if (clear) {
        const uint32_t z = 0;
        Q35CU_CUDA(cudaMemcpyToSymbol(g_device_status, &z, 4));
    }
    uint32_t g = 0, p = 0;
    int rc = gemm_status(&g, clear);
    if (rc) return rc;
    rc = p2p_status(&p, clear);
    if (rc) return rc;
    if (!*status) *status = g ? g : p;
    return Q35CU_OK;
}

}  // namespace q35cu
