// Tensor-core GEMMs of q35_mm_fp8_batch, sm_100a: TMA + tcgen05 + TMEM.
//
// Replaces the CPU loop of q35_mm_fp8_batch (qwen35-c/src/q35_mm.c:158-172)
// for batches of 16 tokens or more.  Y[t, n] = sum_k x[t, k] * e4m3(W[n, k])
// * s[n/128, k/128].  Three kernels, each promoting every 128-column block's
// fp32 partial with its scale in registers:
//   * gemm_e4m3_tc_kernel -- prefill (M >= 128, activations rounded to bf16,
//     the contract: relative L2 <= 5e-3): e4m3 weights x a two-term e4m3
//     split of the activations, block-scaled MMAs (section further down);
//   * gemm_dec_kernel -- multi-token decode, 16..48 tokens of exact fp32
//     activations (the GEMV bound): e4m3 weights x five e4m3 terms per token;
//   * gemm_fp8_tc_kernel (below) -- f16 operands: the weight converted
//     e4m3 -> f16 into TMEM; decode of 49..127 tokens on hi/lo-split fp32
//     activations, and prefill when Q35CU_GEMM_F16 is set.
// Few row tiles (decode): split-K or stream-K, chosen by plan_stream_k.
//
// Roofline: tensor cores for prefill (2*M*N*K flops per launch); HBM for
// decode (each weight byte once per launch).
//
// The f16-operand kernel: both operands f16 on the tensor cores (kind::f16):
//   * every e4m3 value is an f16 value, so a weight tile converts exactly with
//     one cvt.rn.f16x2.e4m3x2 per two elements (bf16 would need four
//     instructions per two: e4m3 -> f16 -> f32 -> bf16);
//   * the activations are prepared once per call (gemm_prep_kernel): each
//     token row is rounded to bf16 and multiplied by 2^-e_t, the power of two
//     that puts its largest magnitude in [2^14, 2^15).  bf16 carries 8
//     significant bits and f16 11, so every element down to 2^-28 of the
//     row's largest converts exactly.  The epilogue multiplies by 2^e_t.
//     Scaling by a power of two commutes with every fp32 rounding in the MMA
//     and in the promotion, so Y equals the bf16 x bf16 computation.
//
// Persistent CTAs (one per SM) walk 128 (weight rows) x 192 (tokens) tiles,
// token tile fastest: the CTAs running together share a few weight row
// blocks (each read from HBM about once) and the activations (L2-resident).
// A call with at most 128 activation rows (multi-token decode on exact
// activations: 2 rows per token) takes a 32-, 64- or 128-row token tile
// instead, so the MMAs, the activation copies and the epilogue cover only
// the rows it has (the weights stream the same way).
//
// Three measured costs shape the kernel:
//   * shared-memory bandwidth: an MMA that reads both operands from shared
//     memory at N = 128 needs all of it, so the converted weight operand
//     never touches shared memory -- the converters write it into TMEM and
//     the MMA reads A from TMEM;
//   * issue: one tcgen05.mma takes ~77 cycles to issue whatever its size,
//     and an N = 128 MMA is only 64 cycles of tensor work, so the tile is
//     N = 192 tokens (96 cycles per MMA) -- P0 | P1 | A0 | A1 then fill
//     the 512 TMEM columns exactly;
//   * barrier waits: a try_wait costs ~120 cycles even on a completed phase,
//     so the MMA warp waits on two barriers per 128-column block (the TMA's
//     bytes on one, the converters and the epilogue on the other -- the
//     TMA's barrier is kept apart so a producer that winds down can wait for
//     its own copies alone) and commits once.
//
// Roles (640 threads; BN = tokens per tile, 192 unless the call is narrower):
//   warp 0      TMA producer of the activation tile [BN tokens x 128 cols]
//               f16 (two 64-column boxes, 128B swizzle), 3 stages;
//   warps 1, 19 lane 0 issues tcgen05.mma kind::f16 (A = the weight tile from
//               TMEM, M = 128; B = the activation tile from shared memory,
//               N = BN; 8 steps of K = 16) into TMEM partial P[g % 2];
//               warp 1 takes the even blocks, warp 19 the odd ones;
//   warp 2      TMA producer of the fp8 weight tile [128 rows x 128 B],
//               4 stages released by the converters;
//   warps 3-6   converters: thread = weight row = TMEM lane; converts its
//               row to f16 and stores it with tcgen05.st into A[g % 2]
//               (64 TMEM columns, two f16 per column along K);
//   warps 7-18  epilogue: warp w owns TMEM lanes 32*(w%4).. (one weight row
//               per thread) and 64 of the BN token columns; it keeps the
//               tile's accumulator in registers, ACC += s[n/128, kb] * P per
//               128-column block (the block scale stays out of the MMA
//               operands, which stay exact), and stores Y after the last block.
//
// Every mbarrier wait is bounded (kWaitNs of wall time).  A wait that gives
// up records Q35CU_ERR_TIMEOUT in the GEMM's device status word (and where:
// role, CTA, block, thread) and raises the CTA's abort flag; every other
// role's wait sees the flag and stops too.  The CTA then winds down so that
// nothing it started can land after it frees its resources:
//   * each producer waits for the copies it issued on barriers only the TMA
//     completes (x_full[], w_full[]), so the wait needs no other role;
//   * each MMA warp commits once more to its own one-shot barrier (fin[]),
//     which fires when every MMA that warp issued has completed;
//   * converters and epilogue warps have nothing in flight (their TMEM
//     stores and loads are waited on where they are made);
// and only then does the CTA pass its final barrier and free TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <atomic>
#include <cstring>

#include "q35cu_internal.h"

namespace q35cu {

__device__ uint32_t g_gemm_status;
// where the first wait that gave up was (role, CTA, block, thread), written
// by the launch that set g_gemm_status
__device__ uint32_t g_gemm_where[4];

namespace {

constexpr int kBM = 128;   // weight rows per tile (MMA M)
constexpr int kBN = 192;   // tokens per tile (MMA N), the widest tile; narrower tiles (BN = 32, 64, 128)
                           // serve calls with fewer activation rows
constexpr int kBK = 128;   // columns per block (one scale block)
// fp8 weight stages (8 stages beside the narrow tiles measured no faster:
// 28-35 us either way for 17408x5120 at 16-64 tokens)
template <int BN> constexpr int wstages() { return 4; }
template <int BN> constexpr uint32_t x_tile() { return BN * kBK * 2; }  // f16 activation tile (48 KB at 192)
constexpr uint32_t kWTile = kBM * kBK;      // 16 KB fp8
template <int BN> constexpr uint32_t x_atom() { return BN * 128; }  // one 64-column swizzle atom of it
// A wait gives up after kWaitNs of wall time (globaltimer) or kWaitIters
// polls, whichever comes first; no wait of a working launch lasts more than
// a few microseconds.
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint32_t kWaitIters = 1u << 28;
// roles recorded with a wait that gave up (g_gemm_where[0])
enum : uint32_t { kRoleX = 1, kRoleW = 2, kRoleMma = 3, kRoleConv = 4, kRoleEpi = 5, kRoleDrain = 6 };
constexpr int kWarpX = 0, kWarpMma = 1, kWarpW = 2, kWarpConv = 3;
constexpr int kConvWarps = 4;                       // one thread per weight row
constexpr int kWarpEpi = kWarpConv + kConvWarps;    // 7
constexpr int kEpiGroups = kBN / 64;                // 64 token columns per epilogue warp (widest tile)
constexpr int kEpiWarps = 4 * kEpiGroups;           // 4 lane quadrants x 3 column groups
constexpr int kWarpMma2 = kWarpEpi + kEpiWarps;     // 19: MMA issuer of the odd blocks
constexpr int kThreads = (kWarpMma2 + 1) * 32;
// Pipeline depth D: TMEM holds D fp32 partials P[0..D) (BN columns each)
// and D converted weight operands A[0..D) (64 columns each: 128 f16 per
// lane); block g uses P[g % D] and A[g % D].  The slot rings (activation
// stages, ready[], done[]) have D + 1 slots.  D = 2 at every tile width:
// D = 4 beside the narrow tiles (room in TMEM) measured no faster.
constexpr uint32_t kACols = kBK / 2;
constexpr uint32_t kTmemCols = 512;
template <int BN> constexpr int depth() { return 2; }
template <int BN> constexpr int stages() { return depth<BN>() + 1; }
template <int BN> constexpr uint32_t tmem_a() { return depth<BN>() * BN; }
static_assert(depth<kBN>() * (kBN + kACols) <= kTmemCols && depth<64>() * (64 + kACols) <= kTmemCols &&
                  depth<128>() * (128 + kACols) <= kTmemCols && depth<32>() * (32 + kACols) <= kTmemCols,
              "TMEM budget");
// arrivals that complete ready[] for block g: the converter warps (A[g % D]
// written) and the epilogue warps (P[g % D] drained of block g - D).  The
// activation tile has its own barrier, x_full[], which only the producer's
// arrive.expect_tx and the TMA's bytes complete.
constexpr uint32_t kStageArrivals = kConvWarps + kEpiWarps;

struct GemmArgs {
    const float *S;       // weight scales [ceil(N/128), kblocks]
    const float *tscale;  // per activation row 2^e_t [m]
    float *Y;             // [m, N] token-major ([m / 2, N] when pair)
    uint32_t N, K, m, kblocks, mtiles, ntiles;
    uint32_t pair;        // rows 2t, 2t+1 are the hi and lo halves of token t: Y[t] = their sum
    // Stream-K (sk == 1; narrow token tiles): the launch's U = ntiles x
    // kblocks (tile, block) units, tile-major, are cut into equal ranges,
    // CTA c taking [U*c/G, U*(c+1)/G), so every CTA converts and multiplies
    // the same number of weight blocks whatever the tile count.  A tile cut
    // by a CTA boundary is finished by segments of several CTAs: each writes
    // its fp32 accumulator to skpart (slot = the tile's first inner boundary
    // c1, segment j = CTA - (c1 - 1)); the CTA whose segment completes the
    // tile's count (skcnt[c1]) adds the segments in order j = 0, 1, ... and
    // stores Y -- a fixed order, so runs repeat bit for bit.
    uint32_t sk;
    uint32_t maxseg;      // segment slots per tile in skpart
    float *skpart;        // [G][maxseg][BN][128] (rows fastest)
    uint32_t *skcnt;      // [G] blocks done of a cut tile (zero between launches)
    uint32_t gm;          // token tiles per raster group (tile_rc); mtiles = one group
};

// The (tile, first block, end block) segments a CTA walks, in order: whole
// tiles blockIdx.x, + gridDim.x, ... or, under stream-K, its unit range.
// SKOK = false compiles the whole-tile walk alone (the 192-token prefill
// tile, whose epilogue has no registers to spare for the stream-K state).
template <bool SKOK>
struct SegWalk {
    uint32_t u, u1, nkb, ntiles, mode, nsplit;
    __device__ __forceinline__ explicit SegWalk(const GemmArgs &a)
        : nkb(a.kblocks), ntiles(a.ntiles), mode(SKOK ? a.sk : 0u), nsplit(a.maxseg)
    {
        if (mode == 1) {  // stream-K: this CTA's range of (tile, block) units
            const uint64_t U = (uint64_t)a.ntiles * a.kblocks;
            u = (uint32_t)(U * blockIdx.x / gridDim.x);
            u1 = (uint32_t)(U * (blockIdx.x + 1) / gridDim.x);
        } else if (mode == 2) {  // split-K: one of a tile's nsplit equal block ranges
            u = blockIdx.x;
            u1 = blockIdx.x < a.ntiles * nsplit ? blockIdx.x + 1 : blockIdx.x;
        } else {
            u = blockIdx.x;
            u1 = a.ntiles;
        }
    }
    __device__ __forceinline__ bool next(uint32_t &tile, uint32_t &kb0, uint32_t &kb1)
    {
        if (u >= u1) return false;
        if (mode == 1) {
            tile = u / nkb;
            kb0 = u % nkb;
            kb1 = nkb - kb0 < u1 - u ? nkb : kb0 + (u1 - u);
            u += kb1 - kb0;
        } else if (mode == 2) {
            tile = u / nsplit;
            const uint32_t part = u % nsplit;
            kb0 = part * nkb / nsplit;
            kb1 = (part + 1) * nkb / nsplit;
            u = u1;
        } else {
            tile = u;
            kb0 = 0;
            kb1 = nkb;
            u += gridDim.x;
        }
        return true;
    }
};

// Where a cut tile's segments meet: the scratch slot, this CTA's segment in
// it and the number of segments.  Stream-K: slot = the tile's first inner
// CTA boundary c1, segment = CTA - (c1 - 1); split-K: slot = the tile,
// segment = its part.
struct SkSlot {
    uint32_t slot, seg, nseg;
};
__device__ __forceinline__ SkSlot sk_slot(const GemmArgs &a, uint32_t tile)
{
    const uint32_t nkb = a.kblocks;
    if (a.sk == 2) return SkSlot{tile, blockIdx.x % a.maxseg, a.maxseg};
    const uint64_t U = (uint64_t)a.ntiles * nkb;
    const uint32_t c1 = (uint32_t)((((uint64_t)tile * nkb + 1) * gridDim.x + U - 1) / U);
    const uint32_t cl = (uint32_t)(((uint64_t)(tile + 1) * nkb * gridDim.x + U - 1) / U) - 1;
    return SkSlot{c1, blockIdx.x + 1 - c1, cl - c1 + 2};
}

// (row block, token tile) of tile index `tile`.  Token tiles are walked in
// groups of gm: inside a group its token tiles go fastest, then the row
// blocks, so the tiles running at once share a band of at most gm token
// tiles -- prepared activations that stay in L2 -- across many weight row
// blocks.  gm == mtiles is one group: token tile fastest over all of them.
__device__ __forceinline__ void tile_rc(uint32_t tile, const GemmArgs &a, uint32_t &rb, uint32_t &mt)
{
    const uint32_t nrb = a.ntiles / a.mtiles;
    const uint32_t span = a.gm * nrb;
    const uint32_t grp = tile / span, in = tile - grp * span;
    const uint32_t g0 = grp * a.gm;
    const uint32_t w = a.mtiles - g0 < a.gm ? a.mtiles - g0 : a.gm;  // token tiles of this group
    rb = in / w;
    mt = g0 + in % w;
}

template <int BN>
struct Smem {  // offsets from the 1024-aligned base (every tile size is a multiple of 1024 B)
    static constexpr uint32_t x(int s) { return s * x_tile<BN>(); }
    static constexpr uint32_t w(int s) { return stages<BN>() * x_tile<BN>() + s * kWTile; }
    static constexpr uint32_t bars = stages<BN>() * x_tile<BN>() + wstages<BN>() * kWTile;
    // x_full, ready, done [S]; w_full, w_empty [WS]; fin [2]; abort flag; TMEM address;
    // stream-K decision word; aborted epilogue warps
    static_assert((3 * stages<BN>() + 2 * wstages<BN>() + 2) * 8 + 16 <= 256, "barriers fit their 256 bytes");
    static constexpr uint32_t total = bars + 256;
    static_assert(x_tile<BN>() % 1024 == 0 && x_atom<BN>() % 1024 == 0, "swizzle atoms need 1024-byte alignment");
};

__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t n)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n));
}
// The producer and MMA roles run with their whole warp converged (so the
// tensor-map, descriptor and TMEM operands are warp-uniform values the
// compiler keeps in uniform registers); the single-thread instructions are
// predicated on `leader` inside the asm rather than branched around.
__device__ __forceinline__ void bar_expect(uint64_t *b, uint32_t bytes, uint32_t leader)
{
    asm volatile(
        "{\n\t.reg .pred e;\n\tsetp.ne.b32 e, %2, 0;\n\t"
        "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(sa(b)),
        "r"(bytes), "r"(leader)
        : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ bool try_wait(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sa(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps (up to ns) until it completes instead of returning at once, so
// waiting warps do not take issue slots from the working ones
__device__ __forceinline__ bool try_wait_sleep(uint64_t *b, uint32_t parity, uint32_t ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(sa(b)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
constexpr uint32_t kSuspendNs = 20000;  // per try: the abort flag and the deadline are checked between tries

__device__ __forceinline__ uint64_t now_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch: a GEMM is launched right after the kernel
// that prepares its activations and may start before that kernel ends; only
// the reads of the prepared activations (and their scales) wait for it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// The slow path of a wait (the phase was not complete at the first poll).
// abort == nullptr: a wind-down wait, which ignores the CTA's abort flag.
__device__ __noinline__ bool bar_wait_slow(uint64_t *b, uint32_t parity, volatile uint32_t *abort, uint32_t role,
                                           uint32_t g)
{
    const uint64_t t0 = now_ns();
    for (uint32_t i = 1; i < kWaitIters; ++i) {
        if (try_wait_sleep(b, parity, kSuspendNs)) return true;
        if (abort && *abort) return false;  // another role gave up: stop without a record of our own
        if (now_ns() - t0 > kWaitNs) break;
    }
    if (abort) *abort = 1;
    if (atomicCAS(&g_gemm_status, 0u, (uint32_t)Q35CU_ERR_TIMEOUT) == 0u) {
        g_gemm_where[0] = role;
        g_gemm_where[1] = blockIdx.x;
        g_gemm_where[2] = g;
        g_gemm_where[3] = threadIdx.x;
    }
    return false;
}

// Bounded wait for phase `parity` of b; false = gave up (or the CTA aborts).
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity, volatile uint32_t *abort, uint32_t role,
                                         uint32_t g)
{
    return try_wait(b, parity) || bar_wait_slow(b, parity, abort, role, g);
}

__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar,
                                       uint32_t leader)
{
    asm volatile(
        "{\n\t.reg .pred e;\n\tsetp.ne.b32 e, %5, 0;\n\t"
        "@e cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        "\n\t}" ::"r"(sa(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(sa(bar)), "r"(leader)
        : "memory");
}

// Wait (bounded, ignoring the abort flag) until the last min(issued, stages)
// copies of a ring have landed.  `full` is completed by the TMA's bytes and
// the producer's own arrive alone, and copy i was issued only after phase
// i - stages of its slot had completed, so phase i is the one pending.
__device__ __forceinline__ void drain(uint64_t *full, int stages, uint32_t issued)
{
    for (uint32_t i = issued > (uint32_t)stages ? issued - stages : 0; i < issued; ++i)
        bar_wait(&full[i % stages], (i / stages) & 1, nullptr, kRoleDrain, i);
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

// kind::f16 instruction descriptor: D f32 (bits 4-5 = 1), A and B f16 (bits
// 7-9 and 10-12 = 0), both K-major, N = BN (bits 17-22 = N/8), M = 128 (bits 24-28 = M/16)
template <int BN>
constexpr uint32_t idesc()
{
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "M = 128 MMAs take N = 16..256 in steps of 16");
    return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem descriptor], issued by the leader lane
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc_,
                                           uint32_t acc, uint32_t leader)
{
    asm volatile(
        "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 e, %5, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc_), "r"(acc), "r"(leader)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t *bar, uint32_t leader)
{
    asm volatile(
        "{\n\t.reg .pred e;\n\tsetp.ne.b32 e, %1, 0;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(sa(bar)),
        "r"(leader)
        : "memory");
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

// four e4m3 bytes (byte 0 first) -> two f16x2 words, exact
__device__ __forceinline__ void e4m3x4_to_f16x4(uint32_t w, uint32_t &lo, uint32_t &hi)
{
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// ACC[i] (+)= s * P[i] for 16 columns; the first block starts the accumulator.
// Packed fma.rn.f32x2 (two independent fp32 FMAs, each rounded as fmaf): in
// the e4m3 kernel, whose epilogue bounds it, 1079 against 999 TFLOP/s with
// scalar FMAs (configuration 2, same box); neutral in the f16 kernel.  The
// first block adds to zero, which leaves the rounded product s * P[i].
__device__ __forceinline__ void promote16(float *acc, const uint32_t (&p)[16], float s, bool first)
{
    uint64_t ss;
    asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint64_t a, pv;
        const float a0 = first ? 0.f : acc[2 * i], a1 = first ? 0.f : acc[2 * i + 1];
        asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
        asm("mov.b64 %0, {%1, %2};" : "=l"(pv) : "r"(p[2 * i]), "r"(p[2 * i + 1]));
        asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(ss), "l"(pv));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[2 * i]), "=f"(acc[2 * i + 1]) : "l"(a));
    }
}

// BN = tokens per tile (the MMA's N): 192 for prefill; 32, 64 or 128 when the
// call has at most that many activation rows, so a multi-token decode call
// moves and multiplies only the columns it has.  Epilogue warps whose 64
// columns lie past BN only take part in the barriers.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                       const __grid_constant__ GemmArgs a)
{
    using Sm = Smem<BN>;
    constexpr int S = stages<BN>(), D = depth<BN>(), WS = wstages<BN>();
    constexpr uint32_t kFull = 0xffffffffu;
    constexpr bool kSK = BN <= 128;  // stream-K is compiled for the narrow token tiles only
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // block g uses slot g % S of the activation rings:
    //   x_full[s]: the activation tile of block g landed (TMA bytes)        -> MMA
    //   ready[s]:  A[g % D] converted + P[g % D] free (converters, epilogue) -> MMA
    //   done[s]:   the MMA of block g completed (tcgen05.commit)           -> all
    // and slot g % WS of the weight ring (w_full: TMA -> converters,
    // w_empty: converters -> TMA).  fin[i]: MMA warp i's last commit.
    uint64_t *x_full = reinterpret_cast<uint64_t *>(sm + Sm::bars);
    uint64_t *ready = x_full + S;
    uint64_t *done = ready + S;
    uint64_t *w_full = done + S;
    uint64_t *w_empty = w_full + WS;
    uint64_t *fin = w_empty + WS;
    volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(fin + 2);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 2) + 1;
    volatile uint32_t *sk_state = reinterpret_cast<volatile uint32_t *>(fin + 2) + 2;
    volatile uint32_t *epi_aborts = reinterpret_cast<volatile uint32_t *>(fin + 2) + 3;

    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t nkb = a.kblocks;
    const uint32_t leader = lane == 0;

    if (warp == kWarpX) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (t == 32) {
        for (int i = 0; i < S; ++i) {
            bar_init(&x_full[i], 1);
            bar_init(&ready[i], kStageArrivals);
            bar_init(&done[i], 1);
        }
        for (int i = 0; i < WS; ++i) {
            bar_init(&w_full[i], 1);
            bar_init(&w_empty[i], kConvWarps);
        }
        bar_init(&fin[0], 1);
        bar_init(&fin[1], 1);
        *abort = 0;
        *epi_aborts = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // Ordering argument for the slot rings (S = D + 1 slots).  Every arrival
    // for block g on a slot of ready[] / x_full[] comes, in its party's
    // program order, after that party waited on done(g - S) (the producer
    // directly, a converter or epilogue thread while handling an earlier
    // block), so the slot has finished its phase for block g - S.  No waiter
    // on done(h) can be overtaken by done(h + S), and no waiter on x_full(h)
    // or ready(h) by phase h + S: each needs that waiter's own later step
    // first.  Every decision to go on or stop is taken warp-wide (__all_sync),
    // so the .sync.aligned TMEM instructions always see a converged warp.
    if (warp == kWarpX) {
        // ---------------- activation producer (whole warp) -----------------
        pdl_wait();  // the prepared activations and scales are complete and visible
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        for (SegWalk<kSK> walk(a); ok && walk.next(tile, kb0, kb1);) {
            uint32_t rb_, mt_;
            tile_rc(tile, a, rb_, mt_);
            const int m0 = (int)(mt_ * BN);
            for (uint32_t kb = kb0; kb < kb1; ++kb, ++g) {
                const int s = g % S;
                if (g >= (uint32_t)S)
                    ok = __all_sync(kFull, bar_wait(&done[s], ((g / S) - 1) & 1, abort, kRoleX, g));
                if (!ok) break;
                bar_expect(&x_full[s], x_tile<BN>(), leader);
                tma_2d(sm + Sm::x(s), &map_x, (int)(kb * kBK), m0, &x_full[s], leader);
                tma_2d(sm + Sm::x(s) + x_atom<BN>(), &map_x, (int)(kb * kBK + 64), m0, &x_full[s], leader);
            }
        }
        drain(x_full, S, g);  // g = copies issued
    } else if (warp == kWarpW) {
        // ---------------- weight producer (whole warp) ---------------------
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        for (SegWalk<kSK> walk(a); ok && walk.next(tile, kb0, kb1);) {
            uint32_t rb_, mt_;
            tile_rc(tile, a, rb_, mt_);
            const int n0 = (int)(rb_ * kBM);
            for (uint32_t kb = kb0; kb < kb1; ++kb, ++g) {
                const int s = g % WS;
                if (g >= (uint32_t)WS)
                    ok = __all_sync(kFull, bar_wait(&w_empty[s], ((g / WS) - 1) & 1, abort, kRoleW, g));
                if (!ok) break;
                bar_expect(&w_full[s], kWTile, leader);
                tma_2d(sm + Sm::w(s), &map_w, (int)(kb * kBK), n0, &w_full[s], leader);
            }
        }
        drain(w_full, WS, g);
    } else if (warp == kWarpMma || warp == kWarpMma2) {
        // ---------------- MMA issuers (whole warp, lane 0 issues) -----------
        // A thread issuing tcgen05.mma blocks until the tensor pipe takes the
        // instruction, so its per-block wait and commit would leave the pipe
        // idle; two warps take alternate blocks (each block has its own P, A
        // and activation stage) and one warp's wait overlaps the other's MMAs.
        const uint32_t parity = warp == kWarpMma ? 0u : 1u;
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        for (SegWalk<kSK> walk(a); ok && walk.next(tile, kb0, kb1);) {
            for (uint32_t kb = kb0; kb < kb1; ++kb, ++g) {
                if ((g & 1) != parity) continue;
                const int s = g % S, j = g % D;
                const uint32_t ph = (g / S) & 1;
                ok = __all_sync(kFull, bar_wait(&x_full[s], ph, abort, kRoleMma, g));
                if (ok) ok = __all_sync(kFull, bar_wait(&ready[s], ph, abort, kRoleMma, g));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t xbase = sa(sm + Sm::x(s));
                const uint32_t d = tmem + j * BN, acol = tmem + tmem_a<BN>() + j * kACols;
#pragma unroll
                for (int ks = 0; ks < kBK / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * x_atom<BN>() + (ks & 3) * 32;
                    mma_f16_ts(d, acol + ks * 8, sw128_desc(xbase + off), idesc<BN>(), ks > 0, leader);
                }
                mma_commit(&done[s], leader);
            }
        }
        // one more commit, to this warp's own barrier: it arrives once every
        // MMA the warp issued has completed (TMEM is freed only after that)
        mma_commit(&fin[parity], leader);
        __syncwarp();
        bar_wait(&fin[parity], 0, nullptr, kRoleDrain, g);
    } else if (warp < kWarpEpi) {
        // ---------------- converters: fp8 -> f16 into TMEM -------------------
        // Thread = weight row = TMEM lane (warp w may access lanes 32*(w%4)..).
        // The 8 lanes of one shared-memory phase (16-byte loads) hold 8
        // consecutive rows, so the swizzled chunk positions (c ^ (r & 7))
        // differ: no bank conflicts.  Column i of A holds K elements 2i, 2i+1.
        const uint32_t quad = warp & 3;
        const uint32_t r = quad * 32 + lane;
        const uint32_t sw = r & 7;
        const uint32_t lane_base = tmem + ((quad * 32) << 16) + tmem_a<BN>();
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        for (SegWalk<kSK> walk(a); ok && walk.next(tile, kb0, kb1);) {
            for (uint32_t kb = kb0; kb < kb1; ++kb, ++g) {
                const int s = g % WS, j = g % D;
                bool w = bar_wait(&w_full[s], (g / WS) & 1, abort, kRoleConv, g);
                // A[g % D] was last read by block g - D
                if (w && g >= (uint32_t)D) w = bar_wait(&done[(g - D) % S], ((g - D) / S) & 1, abort, kRoleConv, g);
                ok = __all_sync(kFull, w);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint8_t *wrow = sm + Sm::w(s) + r * 128;
                uint4 v[8];
#pragma unroll
                for (uint32_t c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint4 *>(wrow + ((c ^ sw) << 4));
                __syncwarp();
                if (lane == 0) bar_arrive(&w_empty[s]);  // the fp8 tile is in registers
#pragma unroll
                for (int hlf = 0; hlf < 2; ++hlf) {
                    uint32_t h[32];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 q = v[hlf * 4 + c];
                        e4m3x4_to_f16x4(q.x, h[8 * c + 0], h[8 * c + 1]);
                        e4m3x4_to_f16x4(q.y, h[8 * c + 2], h[8 * c + 3]);
                        e4m3x4_to_f16x4(q.z, h[8 * c + 4], h[8 * c + 5]);
                        e4m3x4_to_f16x4(q.w, h[8 * c + 6], h[8 * c + 7]);
                    }
                    tmem_st32(lane_base + j * kACols + hlf * 32, h);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(&ready[g % S]);
            }
        }
    } else {
        // ---------------- epilogue: promotion and store -----------------------
        const uint32_t quad = warp & 3;                         // TMEM lanes this warp may touch
        const uint32_t grp = (warp - kWarpEpi) >> 2;            // token columns 64*grp ..
        // columns of this warp inside the tile (all 64 in the widest tile)
        const int ncol = BN == kBN ? 64 : (BN - 64 * (int)grp < 0 ? 0 : (BN - 64 * (int)grp > 64 ? 64 : BN - 64 * (int)grp));
        const uint32_t tbase = tmem + ((quad * 32) << 16) + grp * 64;
        // P[0..D) start out free for blocks 0..D-1
        if (lane == 0)
            for (int i = 0; i < D; ++i) bar_arrive(&ready[i]);
        if constexpr (!kSK) {
            // whole tiles (the 192-token prefill tile)
            uint32_t g = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
                uint32_t rb, mt;
                tile_rc(tile, a, rb, mt);
                const uint32_t n = rb * kBM + quad * 32 + lane;               // weight row
                const uint32_t t0 = mt * BN + grp * 64;                       // first token
                const float *srow = a.S + (size_t)rb * nkb;
                float acc[64];
                float sc = __ldg(srow);
                for (uint32_t kb = 0; kb < nkb; ++kb, ++g) {
                    const int j = g % D;
                    const float sc_next = kb + 1 < nkb ? __ldg(srow + kb + 1) : 0.f;
                    ok = __all_sync(kFull, bar_wait(&done[g % S], (g / S) & 1, abort, kRoleEpi, g));
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (16 * c < ncol) {  // warp-uniform
                            uint32_t p[16];
                            tmem_ld16(tbase + j * BN + c * 16, p);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                            promote16(acc + 16 * c, p, sc, kb == 0);
                        }
                    }
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) bar_arrive(&ready[(g + D) % S]);  // P[g % D] is free for block g + D
                    sc = sc_next;
                }
                if (ok && n < a.N) {
                    if (a.pair) {  // t0 is even: columns (2i, 2i+1) are token (t0 + 2i) / 2's hi and lo
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const uint32_t tok2 = t0 + 2 * i;
                            if (2 * i < ncol && tok2 < a.m)
                                a.Y[(size_t)(tok2 >> 1) * a.N + n] = (acc[2 * i] + acc[2 * i + 1]) * __ldg(a.tscale + tok2);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 64; ++i) {
                            const uint32_t tok = t0 + i;
                            if (i < ncol && tok < a.m) a.Y[(size_t)tok * a.N + n] = acc[i] * __ldg(a.tscale + tok);
                        }
                    }
                }
            }
        } else {
            // the 12 epilogue warps alone (stream-K hand-off of a cut tile)
            auto epi_bar = [] { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); };
            uint32_t g = 0, tile, kb0, kb1;
            bool ok = true;
            // every segment is visited even after an abort: the hand-off of a
            // cut tile needs all 12 warps at its barriers
            for (SegWalk<kSK> walk(a); walk.next(tile, kb0, kb1);) {
                uint32_t rb, mt;
                tile_rc(tile, a, rb, mt);
                const uint32_t row = quad * 32 + lane;
                const uint32_t n = rb * kBM + row;                            // weight row
                const uint32_t t0 = mt * BN + grp * 64;                       // first token
                const float *srow = a.S + (size_t)rb * nkb;
                float acc[64];
                float sc = ok ? __ldg(srow + kb0) : 0.f;
                for (uint32_t kb = kb0; ok && kb < kb1; ++kb, ++g) {
                    const int j = g % D;
                    const float sc_next = kb + 1 < kb1 ? __ldg(srow + kb + 1) : 0.f;
                    ok = __all_sync(kFull, bar_wait(&done[g % S], (g / S) & 1, abort, kRoleEpi, g));
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (16 * c < ncol) {  // warp-uniform
                            uint32_t p[16];
                            tmem_ld16(tbase + j * BN + c * 16, p);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                            promote16(acc + 16 * c, p, sc, kb == kb0);
                        }
                    }
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) bar_arrive(&ready[(g + D) % S]);  // P[g % D] is free for block g + D
                    sc = sc_next;
                }
                bool store = ok;
                if (kSK && (kb0 != 0 || kb1 != nkb)) {
                    // stream-K: this CTA's share of a cut tile.  Slot c1 = the
                    // tile's first inner CTA boundary, segment j = CTA - (c1 - 1).
                    const SkSlot ss = sk_slot(a, tile);
                    float *slot0 = a.skpart + (size_t)ss.slot * a.maxseg * BN * kBM;
                    if (ok) {
                        float *sl = slot0 + (size_t)ss.seg * BN * kBM + (size_t)grp * 64 * kBM + row;
#pragma unroll
                        for (int i = 0; i < 64; ++i)
                            if (i < ncol) sl[(size_t)i * kBM] = acc[i];
                    } else if (lane == 0) {
                        atomicAdd(const_cast<uint32_t *>(epi_aborts), 1u);
                    }
                    epi_bar();
                    if (warp == kWarpEpi && lane == 0) {
                        uint32_t st_ = 0;
                        if (*abort == 0 && *epi_aborts == 0) {
                            __threadfence();
                            const uint32_t done_ = atomicAdd(a.skcnt + ss.slot, kb1 - kb0) + (kb1 - kb0);
                            st_ = 1;
                            if (done_ == nkb) {  // the tile's last segment: this CTA stores it
                                __threadfence();
                                a.skcnt[ss.slot] = 0;  // ready for the next launch
                                st_ = 3;
                            }
                        }
                        *sk_state = st_;
                    }
                    epi_bar();
                    const uint32_t st_ = *sk_state;
                    if (!(st_ & 1)) ok = false;
                    store = (st_ & 2) != 0;
                    if (store) {
                        const float *sl = slot0 + (size_t)grp * 64 * kBM + row;
#pragma unroll
                        for (int i = 0; i < 64; ++i) acc[i] = 0.f;
                        for (uint32_t js = 0; js < ss.nseg; ++js, sl += (size_t)BN * kBM) {
#pragma unroll
                            for (int i = 0; i < 64; ++i)
                                if (i < ncol) acc[i] += __ldcg(sl + (size_t)i * kBM);
                        }
                    }
                }
                if (store && n < a.N) {
                    if (a.pair) {  // t0 is even: columns (2i, 2i+1) are token (t0 + 2i) / 2's hi and lo
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const uint32_t tok2 = t0 + 2 * i;
                            if (2 * i < ncol && tok2 < a.m)
                                a.Y[(size_t)(tok2 >> 1) * a.N + n] = (acc[2 * i] + acc[2 * i + 1]) * __ldg(a.tscale + tok2);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 64; ++i) {
                            const uint32_t tok = t0 + i;
                            if (i < ncol && tok < a.m) a.Y[(size_t)tok * a.N + n] = acc[i] * __ldg(a.tscale + tok);
                        }
                    }
                }
            }
        }
    }

    // Nothing this CTA started is in flight any more: the producers waited
    // for their copies, the MMA warps for their MMAs.
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == kWarpX)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// ---------------------------------------------------------------------------
// Activation preparation: one CTA per token row.  xb = bf16(x) (nearest
// even); e = floor(log2(max |xb|)) - 14, so max |xb| * 2^-e lies in
// [2^14, 2^15) below the f16 limit 65504; Xh = f16(xb * 2^-e), exact for
// every |xb| >= 2^(e-14); tscale = 2^e.  A row of zeros takes e = 0; a row
// whose largest magnitude is infinite or NaN takes e = 0 (the NaN or
// infinity reaches Y as it would in fp32).  e is kept >= -112 so both 2^e
// and 2^-e are normal floats.
// ---------------------------------------------------------------------------
constexpr int kPrepThreads = 256;

template <bool F32>
__device__ __forceinline__ float4 prep_load(const void *x, size_t i4)
{
    if (F32) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i4);
        return make_float4(__bfloat162float(__float2bfloat16_rn(v.x)), __bfloat162float(__float2bfloat16_rn(v.y)),
                           __bfloat162float(__float2bfloat16_rn(v.z)), __bfloat162float(__float2bfloat16_rn(v.w)));
    }
    const uint2 v = __ldg(reinterpret_cast<const uint2 *>(x) + i4);
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                       __uint_as_float(v.y & 0xFFFF0000u));
}

template <bool F32>
__global__ void __launch_bounds__(kPrepThreads) gemm_prep_kernel(const void *X, uint32_t K, uint16_t *Xh,
                                                                 float *tscale)
{
    pdl_trigger();  // the GEMM after this kernel may start streaming weights
    __shared__ float red[kPrepThreads / 32];
    const size_t row = blockIdx.x;
    const uint32_t k4 = K / 4;  // K % 16 == 0
    const size_t base4 = row * k4;
    float mx = 0.f;
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = prep_load<F32>(X, base4 + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kPrepThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    const int eb = (int)((__float_as_uint(mx) >> 23) & 0xFF);
    int e = 0;
    if (eb == 0 && mx > 0.f) e = -112;         // subnormal maximum
    else if (eb > 0 && eb < 255) e = max(eb - 127 - 14, -112);
    const float down = __uint_as_float((uint32_t)(127 - e) << 23);
    uint2 *out = reinterpret_cast<uint2 *>(Xh) + base4;
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = prep_load<F32>(X, base4 + i);
        const __half2 h01 = __floats2half2_rn(v.x * down, v.y * down);
        const __half2 h23 = __floats2half2_rn(v.z * down, v.w * down);
        out[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&h01), *reinterpret_cast<const uint32_t *>(&h23));
    }
    if (threadIdx.x == 0) tscale[row] = __uint_as_float((uint32_t)(127 + e) << 23);
}

// Exact fp32 activations on the tensor cores (the multi-token decode path):
// each token row x (not rounded) is scaled by the power of two 2^-e that
// puts its largest magnitude in [2^14, 2^15) and split into two f16 rows,
// hi = f16(x 2^-e) and lo = f16(x 2^-e - hi) (the difference is exact in
// fp32), so hi + lo carries x to about 22 bits (relative to each element
// down to 2^-28 of the row's largest).  Rows 2t and 2t+1 of Xh; both carry
// tscale = 2^e.
__global__ void __launch_bounds__(kPrepThreads) gemm_prep_split_kernel(const float *X, uint32_t K, uint16_t *Xh,
                                                                       float *tscale)
{
    pdl_trigger();  // the GEMM after this kernel may start streaming weights
    __shared__ float red[kPrepThreads / 32];
    const size_t row = blockIdx.x;
    const uint32_t k4 = K / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(X) + row * k4;
    float mx = 0.f;
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = __ldg(x4 + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kPrepThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    const int eb = (int)((__float_as_uint(mx) >> 23) & 0xFF);
    int e = 0;
    if (eb == 0 && mx > 0.f) e = -112;
    else if (eb > 0 && eb < 255) e = max(eb - 127 - 14, -112);
    const float down = __uint_as_float((uint32_t)(127 - e) << 23);
    uint2 *hi = reinterpret_cast<uint2 *>(Xh) + (2 * row) * k4;
    uint2 *lo = hi + k4;
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = __ldg(x4 + i);
        const float s[4] = {v.x * down, v.y * down, v.z * down, v.w * down};
        __half h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = __float2half_rn(s[j]);
            l[j] = __float2half_rn(s[j] - __half2float(h[j]));
        }
        hi[i] = make_uint2(__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16),
                           __half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16));
        lo[i] = make_uint2(__half_as_ushort(l[0]) | ((uint32_t)__half_as_ushort(l[1]) << 16),
                           __half_as_ushort(l[2]) | ((uint32_t)__half_as_ushort(l[3]) << 16));
    }
    if (threadIdx.x == 0) tscale[2 * row] = tscale[2 * row + 1] = __uint_as_float((uint32_t)(127 + e) << 23);
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

// SMs the persistent GEMM leaves free (q35cu_gemm_reserve_sms)
std::atomic<int> g_gemm_reserved_sms{0};

// SM count of the current device, looked up once per device
int sm_count_of(int dev, int *out)
{
    static int sms[64] = {};
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    if (!sms[dev]) Q35CU_CUDA(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
    *out = sms[dev];
    return Q35CU_OK;
}

}  // namespace

size_t gemm_workspace_bytes(uint32_t m, uint32_t K)
{
    return (((size_t)m * K * 2 + 255) & ~(size_t)255) + (size_t)m * 4;
}

// multi-token decode on the tensor cores with exact fp32 activations: room
// for either preparation -- five e4m3 term rows per token (the default
// kernel) or two f16 rows (the hi/lo kernel) -- with the scales at the end
size_t gemm_exact_workspace_bytes(uint32_t m, uint32_t K)
{
    const size_t terms = (((size_t)m * K * 5 + 255) & ~(size_t)255) + (size_t)m * 4;
    const size_t hilo = gemm_workspace_bytes(2 * m, K);
    return terms > hilo ? terms : hilo;
}

namespace {
// the hi/lo kernel: split prep (2m f16 rows) + the f16 GEMM in pair mode
int launch_gemm_exact_f16(const q35cu_weight *w, const float *X, uint32_t m, float *Y, void *workspace,
                          cudaStream_t st)
{
    if (!m) return Q35CU_OK;
    const uint32_t K = w->cols;
    if (K % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: cols %u not a multiple of 16", K);
    if ((uintptr_t)X % 16 || (uintptr_t)workspace % 16)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned activations or workspace");
    if ((uint64_t)m * 2 > 0x7FFFFFFFu) return set_error(Q35CU_ERR_ARG, "gemm_fp8: too many tokens");
    const size_t need = gemm_exact_workspace_bytes(m, K);
    uint16_t *xh = static_cast<uint16_t *>(workspace);
    float *ts = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + need - (size_t)2 * m * 4);
    gemm_prep_split_kernel<<<m, kPrepThreads, 0, st>>>(X, K, xh, ts);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return launch_gemm_fp8(w, xh, ts, 2 * m, Y, st, true);
}
}  // namespace

int launch_gemm_prep(const void *X, bool f32, uint32_t m, uint32_t K, uint16_t *Xh, float *tscale,
                     cudaStream_t st)
{
    if (!m) return Q35CU_OK;
    if (K % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: cols %u not a multiple of 16", K);
    if ((uintptr_t)X % 16 || (uintptr_t)Xh % 16 || (uintptr_t)tscale % 4)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned activations or workspace");
    if (f32)
        gemm_prep_kernel<true><<<m, kPrepThreads, 0, st>>>(X, K, Xh, tscale);
    else
        gemm_prep_kernel<false><<<m, kPrepThreads, 0, st>>>(X, K, Xh, tscale);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

namespace {

// Token tiles per raster group: the prepared activations of a group (2
// bytes per value in both kernels) within kGroupBytes, so they stay in L2
// while the running tiles sweep the weight row blocks.  Q35CU_GEMM_GROUP
// overrides (0 = one group).
constexpr uint64_t kGroupBytes = (uint64_t)48 << 20;
uint32_t raster_group(uint32_t mtiles, uint32_t bn, uint32_t K)
{
    if (const char *e = getenv("Q35CU_GEMM_GROUP")) {
        const long v = strtol(e, nullptr, 10);
        return v <= 0 || (uint64_t)v >= mtiles ? mtiles : (uint32_t)v;
    }
    const uint64_t per = (uint64_t)bn * K * 2;
    const uint64_t gm = kGroupBytes / per;
    return gm < 1 ? 1u : (gm >= mtiles ? mtiles : (uint32_t)gm);
}

// launch a GEMM kernel as the programmatic dependent of the preparation
// kernel just issued on st
template <typename Kern, typename W>
int launch_after_prep(Kern k, uint32_t grid, uint32_t threads, size_t smem, cudaStream_t st,
                      const CUtensorMap &mx, const W &mw, const GemmArgs &a)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35CU_CUDA(cudaLaunchKernelEx(&cfg, k, mx, mw, a));
    count_launch();
    return Q35CU_OK;
}

// Stream-K scratch, one per device: counters (kSkCntBytes) then the cut
// tiles' partial accumulators.  Grown (never shrunk or freed: CUDA graphs
// may hold its address) when a launch needs more, except under stream
// capture, where such a launch walks whole tiles instead.  Launches on
// different streams of one device that run at the same time must not both
// use it -- the library's own calls run in stream order.
constexpr size_t kSkCntBytes = 4096;
struct SkScratch {
    void *p = nullptr;
    size_t bytes = 0;
};
SkScratch g_sk[64];

// Work split of a launch with few row tiles, fills a's fields (false =
// whole tiles).  Three ways, costed in 128-column block periods of the
// busiest CTA (fitted to B200 timings of multi-token decode: a hand-off of
// a cut tile -- partials out, fence, counter -- ~4.6 periods; each segment
// the tile's finishing CTA adds, ~3; CUDA-graph timing, 16 tokens: `down`
// split-K 31.5 / stream-K 35.6 / whole 52.7 us, 5120x6144 17.8 / 21.3 /
// 22.6, 1024x5120 17.2 (10 parts) / 15.1 / 18.5):
//   whole tiles  ceil(tiles / SMs) * K-blocks;
//   split-K      each tile cut into s = SMs / tiles equal block ranges, one
//                per CTA: ceil(K-blocks / s) + one hand-off + s additions;
//   stream-K     equal (tile, block) unit ranges over G = min(SMs, U / 8)
//                CTAs: a range usually cuts two tiles, so two hand-offs.
// Q35CU_GEMM_SPLIT = whole | split | streamk forces one (comparison).
constexpr uint64_t kSkMinBlocks = 8;             // blocks per CTA at least (amortises a cut tile's hand-off)
constexpr size_t kSkMaxBytes = (size_t)128 << 20;  // scratch cap (48-token e4m3-term tiles: ~91 MB)
constexpr double kHandoff = 4.6, kSegAdd = 3.0;

// cols: accumulator columns a cut tile hands off (BN of the f16 kernel)
bool plan_stream_k(GemmArgs &a, uint32_t cols, uint32_t sms, cudaStream_t st, uint32_t *grid)
{
    if (getenv("Q35CU_GEMM_NO_STREAMK")) return false;
    const char *force = getenv("Q35CU_GEMM_SPLIT");
    const uint64_t nkb = a.kblocks, U = (uint64_t)a.ntiles * nkb;
    const double whole = (double)((a.ntiles + sms - 1) / sms) * nkb;
    double best = whole;
    uint32_t mode = 0, G = 0, maxseg = 0;
    // split-K: at least 4 blocks per part
    const uint64_t s_max = a.ntiles ? sms / a.ntiles : 0;
    const uint64_t s = s_max < nkb / 4 ? s_max : nkb / 4;
    if (s >= 2 && a.ntiles <= kSkCntBytes / 4) {
        const double c = (double)((nkb + s - 1) / s) + kHandoff + kSegAdd * s;
        if (c < best * 0.9) { best = c; mode = 2; G = (uint32_t)(a.ntiles * s); maxseg = (uint32_t)s; }
    }
    const uint32_t Gk = (uint32_t)(U / kSkMinBlocks < sms ? U / kSkMinBlocks : sms);
    if (Gk >= 2) {
        const uint64_t per = U / Gk;
        const uint32_t ms = (uint32_t)((nkb + per - 1) / per + 1);
        const double c = (double)((U + Gk - 1) / Gk) + 2 * kHandoff + kSegAdd * ms;
        if (c < best * 0.9 || (force && !strcmp(force, "streamk"))) { best = c; mode = 1; G = Gk; maxseg = ms; }
    }
    if (force && !strcmp(force, "whole")) mode = 0;
    if (force && !strcmp(force, "split")) {
        if (s >= 2 && a.ntiles <= kSkCntBytes / 4) { mode = 2; G = (uint32_t)(a.ntiles * s); maxseg = (uint32_t)s; }
        else mode = 0;
    }
    if (mode == 0) return false;
    const size_t need = kSkCntBytes + (size_t)(mode == 2 ? a.ntiles : G) * maxseg * cols * kBM * 4;
    if (G * 4 > kSkCntBytes || need > kSkMaxBytes) return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    SkScratch &sc = g_sk[dev];
    if (sc.bytes < need) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) { cudaGetLastError(); return false; }
        if (cs != cudaStreamCaptureStatusNone) return false;
        const size_t bytes = need > ((size_t)16 << 20) ? need : ((size_t)16 << 20);
        void *p = nullptr;
        if (dev_alloc(&p, bytes) != Q35CU_OK) { q35cu_clear_error(); return false; }
        if (cudaMemset(p, 0, kSkCntBytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            cudaGetLastError();
            dev_free(p, bytes);
            return false;
        }
        sc.p = p;  // an earlier, smaller scratch stays allocated (graphs may hold it)
        sc.bytes = bytes;
    }
    a.sk = mode;
    a.maxseg = maxseg;
    *grid = G;
    a.skcnt = static_cast<uint32_t *>(sc.p);
    a.skpart = reinterpret_cast<float *>(static_cast<uint8_t *>(sc.p) + kSkCntBytes);
    return true;
}

template <int BN>
int launch_gemm_bn(const q35cu_weight *w, const uint16_t *Xh, const float *tscale, uint32_t m, float *Y,
                   cudaStream_t st, bool pair)
{
    const uint32_t N = w->rows, K = w->cols;
    const uint64_t mtiles = (m + BN - 1) / BN, ntiles = mtiles * ((N + kBM - 1) / kBM);
    if (ntiles > 0x7FFFFFFFu) return set_error(Q35CU_ERR_ARG, "gemm_fp8: shape too large");
    CUtensorMap mx, mw;
    int rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, Xh, K, m, (uint64_t)K * 2, 64, BN);
    if (rc) return rc;
    rc = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->d_w, K, N, K, 128, kBM);
    if (rc) return rc;
    GemmArgs a{w->d_s, tscale, Y, N, K, m, (K + kBK - 1) / kBK, (uint32_t)mtiles, (uint32_t)ntiles, pair ? 1u : 0u,
               0u, 0u, nullptr, nullptr, 0u};
    a.gm = raster_group((uint32_t)mtiles, BN, K);
    static bool configured[64] = {};  // per instantiation and device
    int dev = 0, sms = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    rc = sm_count_of(dev, &sms);
    if (rc) return rc;
    // leave SMs to kernels that run beside the GEMM (a collective on another stream)
    const int reserve = g_gemm_reserved_sms.load();
    if (reserve > 0 && reserve < sms) sms -= reserve;
    const size_t smem = Smem<BN>::total + 1024;
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(gemm_fp8_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured[dev] = true;
    }
    uint32_t grid = ntiles < (uint64_t)sms ? (uint32_t)ntiles : (uint32_t)sms;
    if (BN <= 128) plan_stream_k(a, BN, (uint32_t)sms, st, &grid);
    return launch_after_prep(gemm_fp8_tc_kernel<BN>, grid, kThreads, smem, st, mx, mw, a);
}

}  // namespace

int launch_gemm_fp8(const q35cu_weight *w, const uint16_t *Xh, const float *tscale, uint32_t m, float *Y,
                    cudaStream_t st, bool pair)
{
    const uint32_t K = w->cols;
    if (!m) return Q35CU_OK;
    if (K % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: cols %u not a multiple of 16", K);
    if (((uintptr_t)Xh % 16) || ((uintptr_t)w->d_w % 16)) return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned operand");
    // the narrowest token tile that holds all m activation rows, up to 128;
    // wider calls take 192-row tiles (the prefill shape)
    if (m <= 32) return launch_gemm_bn<32>(w, Xh, tscale, m, Y, st, pair);
    if (m <= 64) return launch_gemm_bn<64>(w, Xh, tscale, m, Y, st, pair);
    if (m <= 128) return launch_gemm_bn<128>(w, Xh, tscale, m, Y, st, pair);
    return launch_gemm_bn<kBN>(w, Xh, tscale, m, Y, st, pair);
}

// ---------------------------------------------------------------------------
// Prefill GEMM on fp8 operands: tcgen05.mma kind::mxf8f6f4.block_scale,
// e4m3 x e4m3 with UE8M0 scale factors.
//
// The weight tile goes to the tensor cores as the TMA lands it (e4m3, 128
// rows x 128 bytes, 128B swizzle): no conversion, no TMEM operand.  Each
// bf16-valued activation row is carried by two e4m3 terms: with 2^-e
// putting the row's largest magnitude in [2^7, 2^8),
//     x 2^-e = t0 + t1 / 16,  t0 = e4m3(x 2^-e),  t1 = e4m3(16 (x 2^-e - t0)),
// exact for every element of magnitude 2^-6 or more after scaling, so for
// every element down to 2^-13 of the row's largest (below that the error is
// at most 2^-21 of it: half of e4m3's 2^-9 subnormal step in t1, over 16);
// e4m3 keeps 4 significant bits, a bf16 value 8.  The prepared activations
// hold two planes, t0 [m, K] then t1 [m, K].
//
// Each 32-column step of a block is two block-scaled MMAs on the same
// weight slice: one with the t0 tile and B scale factor 2^0, one with the
// t1 tile and scale factor 2^-4 (A's factor is 2^0).  The tensor cores thus
// accumulate W (t0 + t1 / 16) in one fp32 column per token; the scale
// factors are constants, written once into TMEM (every byte of their
// columns, so no layout detail of the factors matters).  The epilogue is the
// f16 kernel's: ACC += s[n/128, kb] * P per 128-column block, Y = ACC * 2^e.
// Against that kernel: no converter warps and no f16 weight in TMEM, the
// same tensor-core time per token (8 fp8 MMAs of K = 32 per block instead of
// 8 f16 MMAs of K = 16) and the same shared-memory bytes per token.
//
// Roles (480 threads), tile 128 weight rows x 192 tokens:
//   warp 0      TMA producer: the t0 and t1 tiles [192 x 128 B each] and the
//               weight tile [128 x 128 B] of a block into one stage, 3 stages;
//   warps 1, 2  lane 0 issues the block's 8 MMAs into TMEM P[g % 2]
//               (192 columns), warp 1 the even blocks, warp 2 the odd ones,
//               and commits to the stage's empty[] and P's tfull[];
//   warps 3-14  epilogue: warp w owns TMEM lanes 32*(w%4).. (one weight row
//               per thread) and 64 of the 192 token columns.
// Waits, abort flag and wind-down as in the f16 kernel: the producer drains
// its copies on TMA-only barriers, each MMA warp waits on its own last
// commit (fin[]), then the CTA frees TMEM.
// ---------------------------------------------------------------------------
namespace {

namespace e4 {
// Tile geometry: BN tokens per tile (MMA N), S stages, D TMEM accumulators,
// EC token columns per epilogue warp (4 * BN / EC epilogue warps); EARLY =
// an epilogue warp loads all its columns, releases the accumulator to the
// MMA, then promotes (else it promotes 32 columns at a time and releases
// after the last).
template <int BN_, int S_, int D_, int EC_, bool EARLY_>
struct Cfg {
    static constexpr int kBN = BN_, kS = S_, kD = D_, kEpiCols = EC_;
    static constexpr bool kEarly = EARLY_;
    static constexpr uint32_t kXTile = kBN * kBK;                // one term plane's tile
    static constexpr uint32_t kStage = 2 * kXTile + kWTile;      // t0, t1, weights
    static constexpr int kWarpMmaA = 1, kWarpMmaB = 2, kWarpEpi0 = 3, kEpiWarps = 4 * kBN / kEpiCols;
    static constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
    static constexpr uint32_t kBars = kS * kStage;
    // TMEM columns: P[0..D) then the scale factors (A reads 4 columns for
    // M = 128, B one per 32 rows of N), 8 columns filled each
    static constexpr uint32_t kSfA = kD * kBN, kSfB0 = kSfA + 8, kSfB1 = kSfB0 + 8;
    static constexpr uint32_t kSmem = kBars + 256;
    // Block-scaled instruction descriptor: B scale-factor byte 0 (bits 4-5),
    // A and B e4m3 (bits 7-9, 10-12 = 0), both K-major, N (bits 17-22 =
    // N/8), scale factors UE8M0 (bit 23), M = 128 (bits 24-28 = M/16), A
    // scale-factor byte 0 (bits 29-30), K = 32 (bit 31 = 0).  D is fp32.
    static constexpr uint32_t kIdesc = ((uint32_t)(kBN >> 3) << 17) | (1u << 23) | ((uint32_t)(kBM >> 4) << 24);
    static_assert(kBN % 16 == 0 && kBN <= 256, "M = 128 MMAs take N = 16..256 in steps of 16");
    static_assert(kBN % kEpiCols == 0 && kEpiCols % 16 == 0, "epilogue columns: whole 16-column loads");
    // full, empty [S]; tfull, tempty [D]; fin [2]; abort flag; TMEM address
    static_assert((2 * kS + 2 * kD + 2) * 8 + 8 <= 256, "barriers fit their 256 bytes");
    static_assert(kSfB1 + 8 <= kTmemCols, "TMEM budget");
    static_assert(kStage % 1024 == 0 && kXTile % 1024 == 0, "swizzle atoms need 1024-byte alignment");
    static_assert(kSmem + 1024 <= 232448, "shared memory");
};
constexpr uint32_t kUe8m0One = 0x7F7F7F7Fu, kUe8m0Sixteenth = 0x7B7B7B7Bu;  // 2^0, 2^-4 in every byte
// 192 tokens, 3 stages, 2 accumulators, 12 epilogue warps of 64 columns.
// Measured slower (configuration-2 projections, same box): 160 tokens with
// 4 stages, 3 accumulators and 20 early-releasing epilogue warps of 32
// columns -- 1034 vs 1067 TFLOP/s at M = 2048, 1053 vs 1110 at M = 8192
// (faster only on gate / up at M = 2048: 1174 vs 1113).
// 16 epilogue warps of 48 columns: 1066-1072 vs 1088-1091 TFLOP/s at
// M = 2048, 1103-1122 vs 1135-1137 at M = 8192 (same box).
using Wide = Cfg<192, 3, 2, 64, false>;

// The weights of one launch: up to kMaxSeg weights with the same K that
// multiply the same activations.  Their row blocks are concatenated --
// segment i owns row blocks [rb0[i], rb0[i+1]) of the launch's tile grid --
// and each has its own tensor map, scales, output and row count, so weights
// that share an input (q | k | v, gate | up) fill the GPU as one GEMM.
constexpr int kMaxSeg = 4;
struct Segs {
    CUtensorMap w[kMaxSeg];
    const float *S[kMaxSeg];  // [ceil(N/128), kblocks]
    float *Y[kMaxSeg];        // [m, N]
    uint32_t N[kMaxSeg];
    uint32_t rb0[kMaxSeg + 1];
    uint32_t nseg;
};
// the segment of launch row block rb: the number of later segments' first
// row blocks at or below it
__device__ __forceinline__ uint32_t seg_of(const Segs &s, uint32_t rb)
{
    uint32_t i = 0;
#pragma unroll
    for (int j = 1; j < kMaxSeg; ++j) i += ((uint32_t)j < s.nseg && rb >= s.rb0[j]) ? 1u : 0u;
    return i;
}
}  // namespace e4

// D[tmem] (+)= (A * sfa)[smem descriptor] * (B * sfb)[smem descriptor], e4m3 x e4m3 -> f32
__device__ __forceinline__ void mma_mx_e4m3(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc_, uint32_t sfa,
                                            uint32_t sfb, uint32_t acc, uint32_t leader)
{
    asm volatile(
        "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %6, 0;\n\tsetp.ne.b32 e, %7, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_), "r"(sfa), "r"(sfb), "r"(acc), "r"(leader)
        : "memory");
}


__device__ __forceinline__ void tmem_st8(uint32_t taddr, uint32_t v)
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
                 : "memory");
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    gemm_e4m3_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ e4::Segs sg,
                        const __grid_constant__ GemmArgs a)
{
    constexpr uint32_t kFull = 0xffffffffu;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // block g: stage g % S (full: TMA bytes landed -> MMA; empty: its MMAs
    // completed -> producer), accumulator g % D (tfull: MMAs completed ->
    // epilogue; tempty: drained by the epilogue warps -> MMA)
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + C::kBars);
    uint64_t *empty = full + C::kS;
    uint64_t *tfull = empty + C::kS;
    uint64_t *tempty = tfull + C::kD;
    uint64_t *fin = tempty + C::kD;
    volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(fin + 2);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 2) + 1;

    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t nkb = a.kblocks;
    const uint32_t leader = lane == 0;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (t == 32) {
        for (int i = 0; i < C::kS; ++i) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], 1);
        }
        for (int i = 0; i < C::kD; ++i) {
            bar_init(&tfull[i], 1);
            bar_init(&tempty[i], C::kEpiWarps);
        }
        bar_init(&fin[0], 1);
        bar_init(&fin[1], 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // the constant scale factors, every byte of their columns, all 128 lanes
    if (warp >= C::kWarpEpi0 && warp < C::kWarpEpi0 + 4) {
        const uint32_t lanes = tmem + (((warp & 3) * 32) << 16);
        tmem_st8(lanes + C::kSfA, e4::kUe8m0One);
        tmem_st8(lanes + C::kSfB0, e4::kUe8m0One);
        tmem_st8(lanes + C::kSfB1, e4::kUe8m0Sixteenth);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    if (warp == 0) {
        // ---------------- producer (whole warp) ------------------------------
        pdl_wait();  // the prepared activations and scales are complete and visible
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < a.ntiles; tile += gridDim.x) {
            uint32_t rb_, mt_;
            tile_rc(tile, a, rb_, mt_);
            const uint32_t si = e4::seg_of(sg, rb_);
            const CUtensorMap *map_w = &sg.w[si];
            const int m0 = (int)(mt_ * C::kBN);
            const int n0 = (int)((rb_ - sg.rb0[si]) * kBM);
            for (uint32_t kb = 0; kb < nkb; ++kb, ++g) {
                const int s = g % C::kS;
                if (g >= (uint32_t)C::kS)
                    ok = __all_sync(kFull, bar_wait(&empty[s], ((g / C::kS) - 1) & 1, abort, kRoleX, g));
                if (!ok) break;
                uint8_t *stage = sm + s * C::kStage;
                bar_expect(&full[s], C::kStage, leader);
                tma_2d(stage, &map_x, (int)(kb * kBK), m0, &full[s], leader);                          // t0
                tma_2d(stage + C::kXTile, &map_x, (int)(kb * kBK), (int)a.m + m0, &full[s], leader);  // t1
                tma_2d(stage + 2 * C::kXTile, map_w, (int)(kb * kBK), n0, &full[s], leader);
            }
        }
        drain(full, C::kS, g);
    } else if (warp == C::kWarpMmaA || warp == C::kWarpMmaB) {
        // ---------------- MMA issuers (whole warp, lane 0 issues) -----------
        const uint32_t parity = warp == C::kWarpMmaA ? 0u : 1u;
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < a.ntiles; tile += gridDim.x) {
            for (uint32_t kb = 0; kb < nkb; ++kb, ++g) {
                if ((g & 1) != parity) continue;
                const int s = g % C::kS, j = g % C::kD;
                ok = __all_sync(kFull, bar_wait(&full[s], (g / C::kS) & 1, abort, kRoleMma, g));
                if (ok && g >= (uint32_t)C::kD)
                    ok = __all_sync(kFull, bar_wait(&tempty[j], ((g / C::kD) - 1) & 1, abort, kRoleMma, g));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t x0 = sa(sm + s * C::kStage), x1 = x0 + C::kXTile, wb = x0 + 2 * C::kXTile;
                const uint32_t d = tmem + j * C::kBN;
#pragma unroll
                for (int ks = 0; ks < kBK / 32; ++ks) {
                    const uint64_t wd = sw128_desc(wb + ks * 32);
                    mma_mx_e4m3(d, wd, sw128_desc(x0 + ks * 32), C::kIdesc, tmem + C::kSfA, tmem + C::kSfB0, ks > 0,
                                leader);
                    mma_mx_e4m3(d, wd, sw128_desc(x1 + ks * 32), C::kIdesc, tmem + C::kSfA, tmem + C::kSfB1, 1,
                                leader);
                }
                mma_commit(&empty[s], leader);
                mma_commit(&tfull[j], leader);
            }
        }
        mma_commit(&fin[parity], leader);
        __syncwarp();
        bar_wait(&fin[parity], 0, nullptr, kRoleDrain, g);
    } else {
        // ---------------- epilogue ----------------------------------------
        const uint32_t quad = warp & 3;                  // TMEM lanes this warp may touch
        const uint32_t grp = (warp - C::kWarpEpi0) >> 2;  // token columns kEpiCols*grp ..
        const uint32_t tbase = tmem + ((quad * 32) << 16) + grp * C::kEpiCols;
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < a.ntiles; tile += gridDim.x) {
            uint32_t rb, mt;
            tile_rc(tile, a, rb, mt);
            const uint32_t si = e4::seg_of(sg, rb);
            const uint32_t lrb = rb - sg.rb0[si], N = sg.N[si];
            float *const Y = sg.Y[si];
            const uint32_t n = lrb * kBM + quad * 32 + lane;         // weight row
            const uint32_t tok0 = mt * C::kBN + grp * C::kEpiCols;  // first token
            const float *srow = sg.S[si] + (size_t)lrb * nkb;
            float acc[C::kEpiCols];
            float sc = __ldg(srow);
            for (uint32_t kb = 0; kb < nkb; ++kb, ++g) {
                const int j = g % C::kD;
                const float sc_next = kb + 1 < nkb ? __ldg(srow + kb + 1) : 0.f;
                ok = __all_sync(kFull, bar_wait(&tfull[j], (g / C::kD) & 1, abort, kRoleEpi, g));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                if constexpr (C::kEarly) {
                    // all of the warp's columns into registers; P[j] goes back
                    // to the MMA before the promotion runs
                    uint32_t p[C::kEpiCols / 16][16];
#pragma unroll
                    for (int c = 0; c < C::kEpiCols / 16; ++c) tmem_ld16(tbase + j * C::kBN + c * 16, p[c]);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) bar_arrive(&tempty[j]);  // P[j] is free for block g + D
#pragma unroll
                    for (int c = 0; c < C::kEpiCols / 16; ++c) promote16(acc + 16 * c, p[c], sc, kb == 0);
                } else {
#pragma unroll
                    for (int c = 0; c < C::kEpiCols / 32; ++c) {  // two loads in flight per wait
                        uint32_t p0[16], p1[16];
                        tmem_ld16(tbase + j * C::kBN + c * 32, p0);
                        tmem_ld16(tbase + j * C::kBN + c * 32 + 16, p1);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        promote16(acc + 32 * c, p0, sc, kb == 0);
                        promote16(acc + 32 * c + 16, p1, sc, kb == 0);
                    }
                    if constexpr (C::kEpiCols % 32 != 0) {  // a last 16 columns
                        constexpr int c0 = C::kEpiCols - 16;
                        uint32_t p0[16];
                        tmem_ld16(tbase + j * C::kBN + c0, p0);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        promote16(acc + c0, p0, sc, kb == 0);
                    }
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) bar_arrive(&tempty[j]);  // P[j] is free for block g + D
                }
                sc = sc_next;
            }
            if (ok && n < N) {
#pragma unroll
                for (int i = 0; i < C::kEpiCols; ++i) {
                    const uint32_t tok = tok0 + i;
                    if (tok < a.m) Y[(size_t)tok * N + n] = acc[i] * __ldg(a.tscale + tok);
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// four floats -> four e4m3 bytes (byte 0 = a), nearest even, saturating
__device__ __forceinline__ uint32_t to_e4m3x4(float a, float b, float c, float d)
{
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
    return lo | (hi << 16);
}

// Activation terms: one CTA per token row.  xb = bf16(x) (nearest even);
// e = floor(log2(max |xb|)) - 7 (kept in [-126, 127]; 0 for a row of zeros
// or one whose largest magnitude is not finite), so max |xb 2^-e| < 2^8 <
// 448, the e4m3 limit.  Row r of plane 0 (Xq[r]): t0 = e4m3(xb 2^-e); row r
// of plane 1 (Xq[m + r]): t1 = e4m3(16 (xb 2^-e - t0)) (the difference and
// the factor are exact in fp32).  A non-finite element becomes the e4m3 NaN
// code (0x7F) in t0 and 0 in t1, so its token's outputs are NaN (an
// infinity included).
template <bool F32>
__global__ void __launch_bounds__(kPrepThreads) gemm_prep_e4m3_kernel(const void *X, uint32_t K, uint32_t m,
                                                                      uint8_t *Xq, float *tscale)
{
    pdl_trigger();  // the GEMM after this kernel may start streaming weights
    __shared__ float red[kPrepThreads / 32];
    const size_t row = blockIdx.x;
    const uint32_t k4 = K / 4;  // K % 16 == 0
    const size_t base4 = row * k4;
    float mx = 0.f;
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = prep_load<F32>(X, base4 + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kPrepThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    const int eb = (int)((__float_as_uint(mx) >> 23) & 0xFF);
    int e = 0;
    if (eb == 0 && mx > 0.f) e = -126;  // subnormal maximum
    else if (eb > 0 && eb < 255) e = max(eb - 127 - 7, -126);
    const float down = __uint_as_float((uint32_t)(127 - e) << 23);
    uint32_t *t0 = reinterpret_cast<uint32_t *>(Xq + row * K);
    uint32_t *t1 = reinterpret_cast<uint32_t *>(Xq + ((size_t)m + row) * K);
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = prep_load<F32>(X, base4 + i);
        const float xs[4] = {v.x * down, v.y * down, v.z * down, v.w * down};
        const uint32_t q0 = to_e4m3x4(xs[0], xs[1], xs[2], xs[3]);
        uint32_t h01, h23;
        e4m3x4_to_f16x4(q0, h01, h23);
        const float2 f01 = __half22float2(*reinterpret_cast<const __half2 *>(&h01));
        const float2 f23 = __half22float2(*reinterpret_cast<const __half2 *>(&h23));
        const float back[4] = {f01.x, f01.y, f23.x, f23.y};
        float r[4];
        uint32_t nan_mask = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const bool fin_ = fabsf(xs[j]) <= 3.402823466e38f;
            r[j] = fin_ ? (xs[j] - back[j]) * 16.f : 0.f;
            if (!fin_) nan_mask |= 0xFFu << (8 * j);
        }
        t0[i] = (q0 & ~nan_mask) | (0x7F7F7F7Fu & nan_mask);
        t1[i] = to_e4m3x4(r[0], r[1], r[2], r[3]);
    }
    if (threadIdx.x == 0) tscale[row] = __uint_as_float((uint32_t)(127 + e) << 23);
}

// One launch over nw weights (1..e4::kMaxSeg) of the same K that multiply
// the prepared activations Xq / tscale: weight i into Y[i] [m, rows_i].
template <class C>
int launch_gemm_e4m3_cfg(const q35cu_weight *const *w, float *const *Y, uint32_t nw, const uint8_t *Xq,
                         const float *tscale, uint32_t m, cudaStream_t st)
{
    if (nw < 1 || nw > (uint32_t)e4::kMaxSeg) return set_error(Q35CU_ERR_ARG, "gemm_fp8: %u weights in one launch", nw);
    const uint32_t K = w[0]->cols;
    const uint64_t mtiles = (m + C::kBN - 1) / C::kBN;
    e4::Segs sg{};
    uint64_t rbs = 0;
    for (uint32_t i = 0; i < nw; ++i) {
        if (w[i]->cols != K) return set_error(Q35CU_ERR_ARG, "gemm_fp8: weights of %u and %u columns", K, w[i]->cols);
        if ((uintptr_t)w[i]->d_w % 16) return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned weight");
        const int rc = make_map(&sg.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w[i]->d_w, K, w[i]->rows, K, 128, kBM);
        if (rc) return rc;
        sg.S[i] = w[i]->d_s;
        sg.Y[i] = Y[i];
        sg.N[i] = w[i]->rows;
        sg.rb0[i] = (uint32_t)rbs;
        rbs += (w[i]->rows + kBM - 1) / kBM;
    }
    sg.nseg = nw;
    for (uint32_t i = nw; i <= (uint32_t)e4::kMaxSeg; ++i) sg.rb0[i] = (uint32_t)rbs;
    const uint64_t ntiles = mtiles * rbs;
    if (ntiles > 0x7FFFFFFFu || (uint64_t)m * 2 > 0x7FFFFFFFu) return set_error(Q35CU_ERR_ARG, "gemm_fp8: shape too large");
    if (!ntiles) return Q35CU_OK;
    CUtensorMap mx;
    int rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, Xq, K, (uint64_t)m * 2, K, 128, C::kBN);
    if (rc) return rc;
    GemmArgs a{nullptr, tscale, nullptr, 0u, K, m, (K + kBK - 1) / kBK, (uint32_t)mtiles, (uint32_t)ntiles, 0u,
               0u, 0u, nullptr, nullptr, 0u};
    a.gm = raster_group((uint32_t)mtiles, C::kBN, K);
    static bool configured[64] = {};  // per configuration and device
    int dev = 0, sms = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    rc = sm_count_of(dev, &sms);
    if (rc) return rc;
    const int reserve = g_gemm_reserved_sms.load();
    if (reserve > 0 && reserve < sms) sms -= reserve;
    const size_t smem = C::kSmem + 1024;
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(gemm_e4m3_tc_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured[dev] = true;
    }
    const uint32_t grid = ntiles < (uint64_t)sms ? (uint32_t)ntiles : (uint32_t)sms;
    return launch_after_prep(gemm_e4m3_tc_kernel<C>, grid, C::kThreads, smem, st, mx, sg, a);
}

int launch_gemm_e4m3(const q35cu_weight *const *w, float *const *Y, uint32_t nw, const uint8_t *Xq,
                     const float *tscale, uint32_t m, cudaStream_t st)
{
    return launch_gemm_e4m3_cfg<e4::Wide>(w, Y, nw, Xq, tscale, m, st);
}

// ---------------------------------------------------------------------------
// Multi-token decode on e4m3 operands (16..127 tokens, exact fp32
// activations): tcgen05.mma kind::f8f6f4, e4m3 x e4m3.
//
// Each fp32 token row x is carried by five e4m3 terms: with 2^-e putting the
// row's largest magnitude in [2^7, 2^8),
//     r0 = x 2^-e,  t_j = e4m3(r_j),  r_{j+1} = 16 (r_j - t_j)
// (every difference and product exact in fp32), so x 2^-e = sum_j t_j 16^-j
// up to the last residual: 1.2e-10 of the row's largest at most (a CPU check
// of the split over N(0, 1) rows; an fp32 value has 24 significant bits, a
// term 4).  Rows 5t .. 5t+4 of the prepared activations are token t's terms,
// so one MMA with N = 5 x tokens multiplies them all with the weight slice as
// the TMA landed it -- no conversion, no TMEM operand.  The epilogue keeps
// the term columns apart through the K loop (ACC += s[n/128, kb] * P per
// 128-column block) and stores Y = (sum_j ACC_j 16^-j) 2^e.
//
// Tiles: 128 weight rows x 16, 32 or 48 tokens (MMA N = 80, 160, 240).
// Stream-K over (tile, 128-column block) units when the row tiles are few,
// as in the f16 kernel: a tile cut by CTA boundaries is finished from its
// segments' accumulators in a fixed order (runs repeat bit for bit).
// Roles: warp 0 producer (a block's activation terms and weight tile into
// one stage), warps 1 and 2 MMA (even / odd blocks; commits release the
// stage and fill the accumulator), warps 3.. epilogue: 4 lane quadrants x
// groups of 16 tokens (80 term columns each).
// ---------------------------------------------------------------------------
namespace dec {
constexpr int kTerms = 5;
constexpr int kTokPerWarp = 16;
constexpr int kColsPerWarp = kTerms * kTokPerWarp;  // 80 term columns per epilogue warp (16-aligned loads)
template <int TOK>
struct Cfg {
    static constexpr int kTok = TOK;                        // tokens per tile
    static constexpr int kN = kTerms * TOK;                 // MMA N
    static constexpr int kGroups = TOK / kTokPerWarp;
    static constexpr int kStride = kN;                      // accumulator column stride
    static constexpr int kD = TOK == 16 ? 4 : (TOK == 32 ? 3 : 2);
    static constexpr uint32_t kXTile = (uint32_t)kN * kBK;
    static constexpr uint32_t kStage = kXTile + kWTile;
    static constexpr int kS = TOK == 16 ? 8 : (TOK == 32 ? 6 : 4);
    static constexpr int kWarpMmaA = 1, kWarpMmaB = 2, kWarpEpi0 = 3, kEpiWarps = 4 * kGroups;
    static constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
    static constexpr uint32_t kBars = kS * kStage;
    static constexpr uint32_t kSmem = kBars + 256;
    static constexpr uint32_t kSkCols = kN;                  // stream-K slot columns
    static_assert(TOK % kTokPerWarp == 0, "whole epilogue groups");
    // kind::f8f6f4: D f32 (bits 4-5 = 1), A and B e4m3 (0), K-major, N, M = 128
    static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
    static_assert(kN % 16 == 0 && kN <= 256, "M = 128 MMAs take N = 16..256 in steps of 16");
    static_assert(kD * kStride <= (int)kTmemCols, "TMEM budget");
    static_assert(kStage % 1024 == 0, "swizzle atoms need 1024-byte alignment");
    static_assert((2 * kS + 2 * kD + 2) * 8 + 16 <= 256, "barriers fit their 256 bytes");
    static_assert(kSmem + 1024 <= 232448, "shared memory");
};
}  // namespace dec

// D[tmem] (+)= A[smem descriptor] * B[smem descriptor], e4m3 x e4m3 -> f32
__device__ __forceinline__ void mma_e4m3_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc_, uint32_t acc,
                                            uint32_t leader)
{
    asm volatile(
        "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 e, %5, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc_), "r"(acc), "r"(leader)
        : "memory");
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    gemm_dec_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                    const __grid_constant__ GemmArgs a)
{
    constexpr uint32_t kFull = 0xffffffffu;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // block g: stage g % S (full: TMA bytes landed -> MMA; empty: its MMAs
    // completed -> producer), accumulator g % D (tfull: MMAs completed ->
    // epilogue; tempty: drained by the epilogue warps -> MMA)
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + C::kBars);
    uint64_t *empty = full + C::kS;
    uint64_t *tfull = empty + C::kS;
    uint64_t *tempty = tfull + C::kD;
    uint64_t *fin = tempty + C::kD;
    volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(fin + 2);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 2) + 1;
    volatile uint32_t *sk_state = reinterpret_cast<volatile uint32_t *>(fin + 2) + 2;
    volatile uint32_t *epi_aborts = reinterpret_cast<volatile uint32_t *>(fin + 2) + 3;

    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t nkb = a.kblocks;
    const uint32_t leader = lane == 0;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (t == 32) {
        for (int i = 0; i < C::kS; ++i) {
            bar_init(&full[i], 1);
            bar_init(&empty[i], 1);
        }
        for (int i = 0; i < C::kD; ++i) {
            bar_init(&tfull[i], 1);
            bar_init(&tempty[i], C::kEpiWarps);
        }
        bar_init(&fin[0], 1);
        bar_init(&fin[1], 1);
        *abort = 0;
        *epi_aborts = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer (whole warp) ------------------------------
        pdl_wait();  // the prepared activations and scales are complete and visible
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        for (SegWalk<true> walk(a); ok && walk.next(tile, kb0, kb1);) {
            uint32_t rb, mt;
            tile_rc(tile, a, rb, mt);
            const int m0 = (int)(mt * C::kN), n0 = (int)(rb * kBM);
            for (uint32_t kb = kb0; kb < kb1; ++kb, ++g) {
                const int s = g % C::kS;
                if (g >= (uint32_t)C::kS)
                    ok = __all_sync(kFull, bar_wait(&empty[s], ((g / C::kS) - 1) & 1, abort, kRoleX, g));
                if (!ok) break;
                uint8_t *stage = sm + s * C::kStage;
                bar_expect(&full[s], C::kStage, leader);
                tma_2d(stage, &map_x, (int)(kb * kBK), m0, &full[s], leader);
                tma_2d(stage + C::kXTile, &map_w, (int)(kb * kBK), n0, &full[s], leader);
            }
        }
        drain(full, C::kS, g);
    } else if (warp == C::kWarpMmaA || warp == C::kWarpMmaB) {
        // ---------------- MMA issuers (whole warp, lane 0 issues) -----------
        const uint32_t parity = warp == C::kWarpMmaA ? 0u : 1u;
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        for (SegWalk<true> walk(a); ok && walk.next(tile, kb0, kb1);) {
            for (uint32_t kb = kb0; kb < kb1; ++kb, ++g) {
                if ((g & 1) != parity) continue;
                const int s = g % C::kS, j = g % C::kD;
                ok = __all_sync(kFull, bar_wait(&full[s], (g / C::kS) & 1, abort, kRoleMma, g));
                if (ok && g >= (uint32_t)C::kD)
                    ok = __all_sync(kFull, bar_wait(&tempty[j], ((g / C::kD) - 1) & 1, abort, kRoleMma, g));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t xb = sa(sm + s * C::kStage), wb = xb + C::kXTile;
                const uint32_t d = tmem + j * C::kStride;
#pragma unroll
                for (int ks = 0; ks < kBK / 32; ++ks)
                    mma_e4m3_ss(d, sw128_desc(wb + ks * 32), sw128_desc(xb + ks * 32), C::kIdesc, ks > 0, leader);
                mma_commit(&empty[s], leader);
                mma_commit(&tfull[j], leader);
            }
        }
        mma_commit(&fin[parity], leader);
        __syncwarp();
        bar_wait(&fin[parity], 0, nullptr, kRoleDrain, g);
    } else {
        // ---------------- epilogue ----------------------------------------
        const uint32_t quad = warp & 3;                      // TMEM lanes this warp may touch
        const uint32_t grp = (warp - C::kWarpEpi0) >> 2;     // tokens 16*grp .. of the tile
        const uint32_t tbase = tmem + ((quad * 32) << 16) + grp * dec::kColsPerWarp;
        const uint32_t row = quad * 32 + lane;
        auto epi_bar = [] { asm volatile("bar.sync 1, %0;" ::"n"(C::kEpiWarps * 32) : "memory"); };
        uint32_t g = 0, tile, kb0, kb1;
        bool ok = true;
        // every segment is visited even after an abort: the hand-off of a cut
        // tile needs all epilogue warps at its barriers
        for (SegWalk<true> walk(a); walk.next(tile, kb0, kb1);) {
            uint32_t rb, mt;
            tile_rc(tile, a, rb, mt);
            const uint32_t n = rb * kBM + row;                                       // weight row
            const uint32_t tok0 = mt * C::kTok + grp * dec::kTokPerWarp;            // first token
            const float *srow = a.S + (size_t)rb * nkb;
            float acc[dec::kColsPerWarp];
            float sc = ok ? __ldg(srow + kb0) : 0.f;
            for (uint32_t kb = kb0; ok && kb < kb1; ++kb, ++g) {
                const int j = g % C::kD;
                const float sc_next = kb + 1 < kb1 ? __ldg(srow + kb + 1) : 0.f;
                ok = __all_sync(kFull, bar_wait(&tfull[j], (g / C::kD) & 1, abort, kRoleEpi, g));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t tcol = tbase + j * C::kStride;
#pragma unroll
                for (int c = 0; c < 2; ++c) {  // two loads in flight per wait
                    uint32_t p0[16], p1[16];
                    tmem_ld16(tcol + c * 32, p0);
                    tmem_ld16(tcol + c * 32 + 16, p1);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    promote16(acc + 32 * c, p0, sc, kb == kb0);
                    promote16(acc + 32 * c + 16, p1, sc, kb == kb0);
                }
                {
                    uint32_t p0[16];
                    tmem_ld16(tcol + 64, p0);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    promote16(acc + 64, p0, sc, kb == kb0);
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) bar_arrive(&tempty[j]);  // the accumulator is free for block g + D
                sc = sc_next;
            }
            bool store = ok;
            if (kb0 != 0 || kb1 != nkb) {
                // stream-K: this CTA's share of a cut tile.  Slot c1 = the
                // tile's first inner CTA boundary, segment = CTA - (c1 - 1).
                const SkSlot ss = sk_slot(a, tile);
                float *slot0 = a.skpart + (size_t)ss.slot * a.maxseg * C::kSkCols * kBM;
                if (ok) {
                    float *sl = slot0 + (size_t)ss.seg * C::kSkCols * kBM + (size_t)grp * dec::kColsPerWarp * kBM + row;
#pragma unroll
                    for (int i = 0; i < dec::kColsPerWarp; ++i) sl[(size_t)i * kBM] = acc[i];
                } else if (lane == 0) {
                    atomicAdd(const_cast<uint32_t *>(epi_aborts), 1u);
                }
                epi_bar();
                if (warp == C::kWarpEpi0 && lane == 0) {
                    uint32_t st_ = 0;
                    if (*abort == 0 && *epi_aborts == 0) {
                        __threadfence();
                        const uint32_t done_ = atomicAdd(a.skcnt + ss.slot, kb1 - kb0) + (kb1 - kb0);
                        st_ = 1;
                        if (done_ == nkb) {  // the tile's last segment: this CTA stores it
                            __threadfence();
                            a.skcnt[ss.slot] = 0;  // ready for the next launch
                            st_ = 3;
                        }
                    }
                    *sk_state = st_;
                }
                epi_bar();
                const uint32_t st_ = *sk_state;
                if (!(st_ & 1)) ok = false;
                store = (st_ & 2) != 0;
                if (store) {
                    const float *sl = slot0 + (size_t)grp * dec::kColsPerWarp * kBM + row;
#pragma unroll
                    for (int i = 0; i < dec::kColsPerWarp; ++i) acc[i] = 0.f;
                    for (uint32_t js = 0; js < ss.nseg; ++js, sl += (size_t)C::kSkCols * kBM) {
#pragma unroll
                        for (int i = 0; i < dec::kColsPerWarp; ++i) acc[i] += __ldcg(sl + (size_t)i * kBM);
                    }
                }
            }
            if (store && n < a.N) {
#pragma unroll
                for (int i = 0; i < dec::kTokPerWarp; ++i) {
                    const uint32_t tok = tok0 + i;
                    if (tok < a.m) {
                        const float *q = acc + dec::kTerms * i;
                        float y = q[4] * 0.0625f + q[3];  // the terms' sum, smallest first: y = q0 + q1/16 + ...
                        y = fmaf(y, 0.0625f, q[2]);
                        y = fmaf(y, 0.0625f, q[1]);
                        y = fmaf(y, 0.0625f, q[0]);
                        a.Y[(size_t)tok * a.N + n] = y * __ldg(a.tscale + tok);
                    }
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// Five e4m3 terms of an exact fp32 token row: one CTA per token.  e =
// floor(log2(max |x|)) - 7 (kept in [-126, 127]; 0 for a row of zeros or one
// whose largest magnitude is not finite); r0 = x 2^-e, t_j = e4m3(r_j),
// r_{j+1} = 16 (r_j - t_j); row 5r + j of Xq holds t_j.  A non-finite
// element becomes the NaN code in t0 and 0 in the other terms.
__global__ void __launch_bounds__(kPrepThreads) gemm_prep_terms_kernel(const float *X, uint32_t K, uint8_t *Xq,
                                                                       float *tscale)
{
    pdl_trigger();  // the GEMM after this kernel may start streaming weights
    __shared__ float red[kPrepThreads / 32];
    const size_t row = blockIdx.x;
    const uint32_t k4 = K / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(X) + row * k4;
    float mx = 0.f;
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = __ldg(x4 + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kPrepThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    const int eb = (int)((__float_as_uint(mx) >> 23) & 0xFF);
    int e = 0;
    if (eb == 0 && mx > 0.f) e = -126;
    else if (eb > 0 && eb < 255) e = max(eb - 127 - 7, -126);
    const float down = __uint_as_float((uint32_t)(127 - e) << 23);
    uint32_t *out = reinterpret_cast<uint32_t *>(Xq + dec::kTerms * row * K);
    for (uint32_t i = threadIdx.x; i < k4; i += kPrepThreads) {
        const float4 v = __ldg(x4 + i);
        float r[4] = {v.x * down, v.y * down, v.z * down, v.w * down};
        uint32_t nan_mask = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (!(fabsf(r[q]) <= 3.402823466e38f)) {
                nan_mask |= 0xFFu << (8 * q);
                r[q] = 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < dec::kTerms; ++j) {
            const uint32_t tq = to_e4m3x4(r[0], r[1], r[2], r[3]);
            out[(size_t)j * k4 + i] = j == 0 ? (tq & ~nan_mask) | (0x7F7F7F7Fu & nan_mask) : tq;
            if (j + 1 < dec::kTerms) {
                uint32_t h01, h23;
                e4m3x4_to_f16x4(tq, h01, h23);
                const float2 f01 = __half22float2(*reinterpret_cast<const __half2 *>(&h01));
                const float2 f23 = __half22float2(*reinterpret_cast<const __half2 *>(&h23));
                r[0] = (r[0] - f01.x) * 16.f;
                r[1] = (r[1] - f01.y) * 16.f;
                r[2] = (r[2] - f23.x) * 16.f;
                r[3] = (r[3] - f23.y) * 16.f;
            }
        }
    }
    if (threadIdx.x == 0) tscale[row] = __uint_as_float((uint32_t)(127 + e) << 23);
}

template <class C>
int launch_gemm_dec_cfg(const q35cu_weight *w, const uint8_t *Xq, const float *tscale, uint32_t m, float *Y,
                        cudaStream_t st)
{
    const uint32_t N = w->rows, K = w->cols;
    const uint64_t mtiles = (m + C::kTok - 1) / C::kTok, ntiles = mtiles * ((N + kBM - 1) / kBM);
    if (ntiles > 0x7FFFFFFFu) return set_error(Q35CU_ERR_ARG, "gemm_fp8: shape too large");
    CUtensorMap mx, mw;
    // the term rows of every token tile: mtiles * kN rows (the last tile's
    // rows past 5m read zeros)
    int rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, Xq, K, (uint64_t)m * dec::kTerms, K, 128, C::kN);
    if (rc) return rc;
    rc = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->d_w, K, N, K, 128, kBM);
    if (rc) return rc;
    GemmArgs a{w->d_s, tscale, Y, N, K, m, (K + kBK - 1) / kBK, (uint32_t)mtiles, (uint32_t)ntiles, 0u,
               0u, 0u, nullptr, nullptr, 0u};
    a.gm = (uint32_t)mtiles;  // token tile fastest: a row block's token tiles share its weight stream
    static bool configured[64] = {};  // per configuration and device
    int dev = 0, sms = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    rc = sm_count_of(dev, &sms);
    if (rc) return rc;
    const int reserve = g_gemm_reserved_sms.load();
    if (reserve > 0 && reserve < sms) sms -= reserve;
    const size_t smem = C::kSmem + 1024;
    if (!configured[dev]) {
        Q35CU_CUDA(cudaFuncSetAttribute(gemm_dec_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured[dev] = true;
    }
    uint32_t grid = ntiles < (uint64_t)sms ? (uint32_t)ntiles : (uint32_t)sms;
    plan_stream_k(a, C::kSkCols, (uint32_t)sms, st, &grid);
    return launch_after_prep(gemm_dec_kernel<C>, grid, C::kThreads, smem, st, mx, mw, a);
}

// the f16 hi/lo kernel for multi-token decode when Q35CU_GEMV_TC_F16 is set
bool dec_use_f16() { return getenv("Q35CU_GEMV_TC_F16") != nullptr; }
constexpr uint32_t kDecMaxTokens = 48;  // larger batches take the hi/lo kernel

// the fp8-operand kernel unless Q35CU_GEMM_F16 asks for the f16 one
bool use_e4m3() { return getenv("Q35CU_GEMM_F16") == nullptr; }

// preparation into acts (2 m K bytes) and ts (m scales), then the GEMM of
// nw weights with the same K: weight i into Y[i]
int gemm_bf16_multi_into(const q35cu_weight *const *w, float *const *Y, uint32_t nw, const void *X, bool f32,
                         uint32_t m, void *acts, float *ts, cudaStream_t st)
{
    const uint32_t K = w[0]->cols;
    if (K % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: cols %u not a multiple of 16", K);
    if ((uintptr_t)X % 16 || (uintptr_t)acts % 16 || (uintptr_t)ts % 4)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned activations or workspace");
    for (uint32_t i = 0; i < nw; ++i) {
        if (w[i]->cols != K) return set_error(Q35CU_ERR_ARG, "gemm_fp8: weights of %u and %u columns", K, w[i]->cols);
        if ((uintptr_t)w[i]->d_w % 16) return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned weight");
    }
    if (!use_e4m3()) {  // one preparation, a launch per weight
        uint16_t *xh = static_cast<uint16_t *>(acts);
        int rc = launch_gemm_prep(X, f32, m, K, xh, ts, st);
        for (uint32_t i = 0; !rc && i < nw; ++i) rc = launch_gemm_fp8(w[i], xh, ts, m, Y[i], st);
        return rc;
    }
    uint8_t *xq = static_cast<uint8_t *>(acts);
    if (f32)
        gemm_prep_e4m3_kernel<true><<<m, kPrepThreads, 0, st>>>(X, K, m, xq, ts);
    else
        gemm_prep_e4m3_kernel<false><<<m, kPrepThreads, 0, st>>>(X, K, m, xq, ts);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return launch_gemm_e4m3(w, Y, nw, xq, ts, m, st);
}

int gemm_bf16_into(const q35cu_weight *w, const void *X, bool f32, uint32_t m, float *Y, void *acts, float *ts,
                   cudaStream_t st)
{
    return gemm_bf16_multi_into(&w, &Y, 1, X, f32, m, acts, ts, st);
}

}  // namespace

// Prefill GEMM on bf16-valued activations (X bf16 bits, or fp32 rounded to
// bf16 when f32): prepares the activations into `workspace`
// (gemm_workspace_bytes(m, K): 2 m K bytes of prepared values, then m
// scales) and runs the tensor-core GEMM.
int launch_gemm_exact(const q35cu_weight *w, const float *X, uint32_t m, float *Y, void *workspace,
                      cudaStream_t st)
{
    if (!m) return Q35CU_OK;
    // e4m3 terms up to 48 tokens; above, two f16 rows per token beat five
    // e4m3 rows (CUDA-graph timing, 17408x5120: 16 / 32 / 48 tokens 22.6 /
    // 27.6 / 35.6 us against 25.6 / 32.4 / 37.3; 64 / 100 tokens 44.7 / 84.7
    // against 37.3 / 64.0)
    if (m > kDecMaxTokens || dec_use_f16()) return launch_gemm_exact_f16(w, X, m, Y, workspace, st);
    const uint32_t K = w->cols;
    if (K % 16) return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: cols %u not a multiple of 16", K);
    if ((uintptr_t)X % 16 || (uintptr_t)workspace % 16 || (uintptr_t)w->d_w % 16)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8: misaligned activations, weight or workspace");
    if ((uint64_t)m * dec::kTerms > 0x7FFFFFFFu) return set_error(Q35CU_ERR_ARG, "gemm_fp8: too many tokens");
    const size_t need = gemm_exact_workspace_bytes(m, K);
    uint8_t *xq = static_cast<uint8_t *>(workspace);
    float *ts = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + need - (size_t)m * 4);
    gemm_prep_terms_kernel<<<m, kPrepThreads, 0, st>>>(X, K, xq, ts);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    // one token tile of 16, 32 or 48
    if (m <= 16) return launch_gemm_dec_cfg<dec::Cfg<16>>(w, xq, ts, m, Y, st);
    if (m <= 32) return launch_gemm_dec_cfg<dec::Cfg<32>>(w, xq, ts, m, Y, st);
    return launch_gemm_dec_cfg<dec::Cfg<48>>(w, xq, ts, m, Y, st);
}

int launch_gemm_bf16(const q35cu_weight *w, const void *X, bool f32, uint32_t m, float *Y, void *workspace,
                     cudaStream_t st)
{
    if (!m) return Q35CU_OK;
    const size_t need = gemm_workspace_bytes(m, w->cols);
    float *ts = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + need - (size_t)m * 4);
    return gemm_bf16_into(w, X, f32, m, Y, workspace, ts, st);
}

int launch_gemm_bf16_multi(const q35cu_weight *const *w, float *const *Y, uint32_t nw, const void *X, bool f32,
                           uint32_t m, void *workspace, cudaStream_t st)
{
    if (!m) return Q35CU_OK;
    const size_t need = gemm_workspace_bytes(m, w[0]->cols);
    float *ts = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + need - (size_t)m * 4);
    return gemm_bf16_multi_into(w, Y, nw, X, f32, m, workspace, ts, st);
}

// ---------------------------------------------------------------------------
// Prefill GEMM for callers that must not allocate device memory.
//
// q35cu_gemm_fp8 takes a caller-provided workspace for the prepared (f16,
// per-token scaled) copy of the activations, and the host entry point
// q35_mm_fp8_batch keeps that copy in a buffer it allocates.  Some callers
// can do neither at that point: a serving process that reserved its whole
// HBM budget up front, or a decode/prefill loop that cannot afford the
// device-wide synchronisation a cudaMalloc/cudaFree may imply.  For them the
// prepared copy lives in fixed arrays compiled into this file instead.
//
//   * the arrays hold kNoAllocMaxActs f16 values (16 MiB) and one scale per
//     token (2 MiB: cols is a multiple of 16, so m <= kNoAllocMaxActs / 16);
//     every GPU that loads the library keeps them until the process exits;
//   * a call with m * cols > kNoAllocMaxActs is rejected with Q35CU_ERR_ARG;
//   * every call reuses the same arrays: two calls whose work overlaps on the
//     GPU (different streams, no ordering) race on them;
//   * each call overwrites exactly the m * cols values and m scales it reads,
//     so nothing needs clearing between calls;
//   * the first call on a device looks up the arrays' device addresses
//     (cudaGetSymbolAddress) and sets the GEMM's shared-memory limit; make
//     that first call before any stream capture.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocMaxActs = (size_t)8 << 20;
static __device__ __align__(256) uint16_t g_noalloc_acts[kNoAllocMaxActs];
static __device__ __align__(256) float g_noalloc_tscale[kNoAllocMaxActs / 16];

namespace {

// the arrays' device addresses, looked up once per device with that device current
int noalloc_scratch(uint16_t **acts, float **tscale)
{
    static uint16_t *a_addr[64] = {};
    static float *s_addr[64] = {};
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(Q35CU_ERR_NODEV, "device %d", dev);
    if (!a_addr[dev]) {
        void *p = nullptr, *q = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_acts);
        if (e != cudaSuccess || !p) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_acts)");
        e = cudaGetSymbolAddress(&q, g_noalloc_tscale);
        if (e != cudaSuccess || !q) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_tscale)");
        s_addr[dev] = static_cast<float *>(q);
        a_addr[dev] = static_cast<uint16_t *>(p);
    }
    *acts = a_addr[dev];
    *tscale = s_addr[dev];
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
    uint16_t *xh = nullptr;
    float *ts = nullptr;
    int rc = noalloc_scratch(&xh, &ts);
    if (rc) return rc;
    return gemm_bf16_into(w, X, true, m, Y, xh, ts, st);
}

int gemm_reserve_sms(int n)
{
    if (n < 0) return set_error(Q35CU_ERR_ARG, "gemm_reserve_sms: %d", n);
    g_gemm_reserved_sms.store(n);
    return Q35CU_OK;
}

uint32_t *gemm_status_word()
{
    void *p = nullptr;
    return cudaGetSymbolAddress(&p, g_gemm_status) == cudaSuccess ? static_cast<uint32_t *>(p) : nullptr;
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

// where the wait that set the status gave up (kept until the next one does)
int gemm_timeout_info(uint32_t out[4])
{
    Q35CU_CUDA(cudaMemcpyFromSymbol(out, g_gemm_where, 4 * sizeof(uint32_t)));
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
