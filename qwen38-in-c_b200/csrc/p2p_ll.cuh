// The peer-memory word protocol shared by the standalone collectives
// (p2p.cu) and the GEMV's tensor-parallel epilogue (gemv.cu).
//
// Every rank owns an exchange area in its HBM, mapped into every other rank's
// process (CUDA IPC).  A value travels as one 8-byte word {value, sequence
// number}; an aligned 8-byte store is seen whole or not at all, so a receiver
// polls its own area until the word carries the current sequence number.
// Area layout (bytes):
//   [0, 4)      sequence number of the last collective (local)
//   [4, 8)      CTAs of the current collective that finished (local)
//   [4096, ..)  words: [2 sets][kP2PMaxRanks ranks][kP2PMaxElems]
// Collective number s uses set s & 1.
#pragma once

#include <cstdint>

namespace q35cu {

constexpr int kP2PMaxRanks = 8;
constexpr size_t kP2PMaxElems = 256 * 1024;
constexpr size_t kP2PSeqOff = 0;
constexpr size_t kP2PTicketOff = 4;
constexpr size_t kP2PDataOff = 4096;
constexpr size_t kP2PAreaBytes = kP2PDataOff + 2 * kP2PMaxRanks * kP2PMaxElems * 8;
constexpr uint32_t kP2PSpinLimit = 1u << 24;

// every rank's exchange area as mapped in this process
struct P2PView {
    uint8_t *area[kP2PMaxRanks];
    int rank, world;
};

__device__ __forceinline__ uint64_t *p2p_slot(uint8_t *area, uint32_t seq, int src)
{
    return reinterpret_cast<uint64_t *>(area + kP2PDataOff) + ((size_t)(seq & 1) * kP2PMaxRanks + src) * kP2PMaxElems;
}
__device__ __forceinline__ void p2p_put(uint64_t *p, float v, uint32_t seq)
{
    const uint64_t w = (uint64_t)__float_as_uint(v) | ((uint64_t)seq << 32);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// the value of word p once it carries `seq`; a wait that gives up stores
// Q35CU_ERR_TIMEOUT (7) in *status and returns what the word holds
__device__ __forceinline__ float p2p_get(const uint64_t *p, uint32_t seq, uint32_t *status)
{
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    for (uint32_t i = 0; (uint32_t)(w >> 32) != seq; ++i) {
        if (i >= kP2PSpinLimit) {
            atomicExch(status, 7u);
            break;
        }
        if (i > 32) __nanosleep(32);
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    }
    return __uint_as_float((uint32_t)w);
}
// this collective's sequence number (read by one thread once the previous
// kernel completed; every CTA of the collective reads the same value)
__device__ __forceinline__ uint32_t p2p_next_seq(const P2PView &v)
{
    return *reinterpret_cast<volatile uint32_t *>(v.area[v.rank] + kP2PSeqOff) + 1;
}
// called by one thread per CTA at the very end: the last CTA to finish
// advances the sequence number for the next collective
__device__ __forceinline__ void p2p_finish(const P2PView &v, uint32_t seq)
{
    uint8_t *mine = v.area[v.rank];
    uint32_t *ticket = reinterpret_cast<uint32_t *>(mine + kP2PTicketOff);
    __threadfence();
    if (atomicAdd(ticket, 1u) == gridDim.x * gridDim.y - 1) {
        *ticket = 0;
        *reinterpret_cast<volatile uint32_t *>(mine + kP2PSeqOff) = seq;
        __threadfence();
    }
}

}  // namespace q35cu
