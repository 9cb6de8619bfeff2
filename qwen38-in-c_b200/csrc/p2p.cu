// Tensor-parallel collectives over NVLink peer memory (one process per GPU).
//
// The decode step of a tensor-parallel stack exchanges small vectors between
// projections: the row-parallel outputs (out/o/down, qwen35-c/src/q35_model.c
// and q35_deltanet.c, 5120 fp32) are summed across ranks and the
// column-parallel outputs (gate/up/qkv/z/q/k/v) are gathered.  A library
// collective call for such a vector costs several microseconds of fixed
// latency and a step makes 128-256 of them, so these one-shot collectives move
// the data with plain stores into the peers' memory instead:
//
//   * every rank owns an exchange area in its HBM (allocated here, shared with
//     the other processes through CUDA IPC handles the caller passes around);
//   * each value travels as one 8-byte word {value, sequence number}: CTA c
//     stores its chunk into slot[rank] of every rank's area (NVLink stores to
//     the peers), and the receiver polls the words of its own area until each
//     carries the current sequence number -- an aligned 8-byte store is seen
//     whole or not at all, so no fence or separate flag is needed and the
//     data crosses NVLink once;
//   * the values are combined in rank order -- the sum is the same on every
//     rank and from run to run (no atomics);
//   * the sequence number of a collective lives in device memory (every CTA
//     reads it after the previous kernel completed, the last CTA to finish
//     advances it), so a CUDA graph that replays the collective stays in
//     step and no word left by an earlier collective -- whatever its length
//     and chunking -- carries the current number; two buffer sets
//     alternate, so a rank that runs ahead never overwrites data a slower
//     rank has not read yet (it cannot run two collectives ahead: the second
//     needs the slower rank's data of the first).
//
// The kernels take part in programmatic dependent launch: the next kernel may
// start its own prologue while a collective waits for its peers.
//
// A wait that gives up records Q35CU_ERR_TIMEOUT in the device status word
// (q35cu_device_status) and the kernel finishes without the missing data.
#include <cuda_runtime.h>

#include <cstring>

#include "p2p_ll.cuh"
#include "q35cu_internal.h"

namespace q35cu {

// bounded waits of the collectives that gave up (read by device_status)
__device__ uint32_t g_p2p_status;

namespace {

constexpr int kMaxChunks = 32;  // CTAs per collective
constexpr uint32_t kThreads = 256;

// push this CTA's chunk src[lo, hi) into slot[rank] of every area; returns
// the collective's sequence number
__device__ __forceinline__ uint32_t push(const P2PView &a, const float *src, uint32_t lo, uint32_t hi)
{
    __shared__ uint32_t s_seq;
    if (threadIdx.x == 0) s_seq = p2p_next_seq(a);
    __syncthreads();
    const uint32_t seq = s_seq;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += kThreads) {
        const float v = src[i];
        for (int d = 0; d < a.world; ++d) p2p_put(p2p_slot(a.area[d], seq, a.rank) + i, v, seq);
    }
    return seq;
}

__global__ void __launch_bounds__(kThreads) p2p_allreduce_kernel(const __grid_constant__ P2PView a, const float *in,
                                                                 float *out, uint32_t n)
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // `in` is the previous kernel's output
    const uint32_t lo = (uint32_t)(((uint64_t)blockIdx.x * n) / gridDim.x);
    const uint32_t hi = (uint32_t)(((uint64_t)(blockIdx.x + 1) * n) / gridDim.x);
    const uint32_t seq = push(a, in, lo, hi);
    __syncthreads();  // every read of `in` by this CTA is done before `out` (may alias) is written
    uint8_t *mine = a.area[a.rank];
    for (uint32_t i = lo + threadIdx.x; i < hi; i += kThreads) {
        float v = 0.f;
        for (int s = 0; s < a.world; ++s) v += p2p_get(p2p_slot(mine, seq, s) + i, seq, &g_p2p_status);  // rank order
        out[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) p2p_finish(a, seq);
}

__global__ void __launch_bounds__(kThreads) p2p_allgather_kernel(const __grid_constant__ P2PView a, const float *send,
                                                                 float *recv, uint32_t n)
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t lo = (uint32_t)(((uint64_t)blockIdx.x * n) / gridDim.x);
    const uint32_t hi = (uint32_t)(((uint64_t)(blockIdx.x + 1) * n) / gridDim.x);
    const uint32_t seq = push(a, send, lo, hi);
    uint8_t *mine = a.area[a.rank];
    for (int s = 0; s < a.world; ++s)
        for (uint32_t i = lo + threadIdx.x; i < hi; i += kThreads)
            recv[(size_t)s * n + i] = p2p_get(p2p_slot(mine, seq, s) + i, seq, &g_p2p_status);
    __syncthreads();
    if (threadIdx.x == 0) p2p_finish(a, seq);
}

struct P2PState {
    int device = -1;
    uint8_t *own = nullptr;
    P2PView args{};
    bool open = false;
};
P2PState g_p2p;

template <typename Kern>
int launch_p2p(Kern k, uint32_t grid, cudaStream_t st, const float *a, float *b, uint32_t n)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q35CU_CUDA(cudaLaunchKernelEx(&cfg, k, g_p2p.args, a, b, n));
    count_launch();
    return Q35CU_OK;
}

uint32_t chunks_for(size_t n)
{
    const size_t c = (n + 255) / 256;
    return (uint32_t)(c < 1 ? 1 : (c > (size_t)kMaxChunks ? kMaxChunks : c));
}

}  // namespace

bool p2p_view(P2PView *out)
{
    if (!g_p2p.open) return false;
    *out = g_p2p.args;
    return true;
}

uint32_t *p2p_status_word()
{
    void *p = nullptr;
    return cudaGetSymbolAddress(&p, g_p2p_status) == cudaSuccess ? static_cast<uint32_t *>(p) : nullptr;
}

int p2p_status(uint32_t *status, bool clear)
{
    Q35CU_CUDA(cudaMemcpyFromSymbol(status, g_p2p_status, 4));
    if (clear) {
        const uint32_t z = 0;
        Q35CU_CUDA(cudaMemcpyToSymbol(g_p2p_status, &z, 4));
    }
    return Q35CU_OK;
}

}  // namespace q35cu

using namespace q35cu;

#define Q35_API extern "C" __attribute__((visibility("default")))

Q35_API size_t q35cu_p2p_max_elems(void) { return kP2PMaxElems; }

Q35_API int q35cu_p2p_handle(void *out, size_t cap)
{
    if (!out || cap < sizeof(cudaIpcMemHandle_t))
        return set_error(Q35CU_ERR_ARG, "p2p handle needs %zu bytes", sizeof(cudaIpcMemHandle_t));
    int dev = 0;
    Q35CU_CUDA(cudaGetDevice(&dev));
    if (g_p2p.own && g_p2p.device != dev)
        return set_error(Q35CU_ERR_ARG, "p2p exchange area belongs to device %d, not %d", g_p2p.device, dev);
    if (!g_p2p.own) {
        void *p = nullptr;
        Q35CU_CUDA(cudaMalloc(&p, kP2PAreaBytes));
        // sequence numbers and words start at zero (no word carries a live
        // sequence number) before any peer can see the area
        cudaError_t e = cudaMemset(p, 0, kP2PAreaBytes);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            cudaFree(p);
            return cuda_error(e, "p2p exchange area");
        }
        g_p2p.own = static_cast<uint8_t *>(p);
        g_p2p.device = dev;
    }
    cudaIpcMemHandle_t h;
    Q35CU_CUDA(cudaIpcGetMemHandle(&h, g_p2p.own));
    memcpy(out, &h, sizeof(h));
    return Q35CU_OK;
}

Q35_API int q35cu_p2p_open(int rank, int world, const void *handles, size_t handle_bytes)
{
    if (world < 1 || world > kP2PMaxRanks || rank < 0 || rank >= world || !handles ||
        handle_bytes < sizeof(cudaIpcMemHandle_t))
        return set_error(Q35CU_ERR_ARG, "p2p_open: rank %d world %d", rank, world);
    if (!g_p2p.own) return set_error(Q35CU_ERR_ARG, "p2p_open: call q35cu_p2p_handle first");
    if (g_p2p.open) return set_error(Q35CU_ERR_ARG, "p2p_open: already open");
    P2PView a{};
    a.rank = rank;
    a.world = world;
    for (int r = 0; r < world; ++r) {
        if (r == rank) {
            a.area[r] = g_p2p.own;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * handle_bytes, sizeof(h));
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != rank && a.area[q]) cudaIpcCloseMemHandle(a.area[q]);
            return cuda_error(e, "cudaIpcOpenMemHandle");
        }
        a.area[r] = static_cast<uint8_t *>(p);
    }
    g_p2p.args = a;
    g_p2p.open = true;
    return Q35CU_OK;
}

Q35_API int q35cu_p2p_close(void)
{
    int rc = Q35CU_OK;
    if (g_p2p.open) {
        for (int r = 0; r < g_p2p.args.world; ++r)
            if (r != g_p2p.args.rank && g_p2p.args.area[r]) {
                const cudaError_t e = cudaIpcCloseMemHandle(g_p2p.args.area[r]);
                if (e != cudaSuccess && rc == Q35CU_OK) rc = cuda_error(e, "cudaIpcCloseMemHandle");
            }
        g_p2p.open = false;
        g_p2p.args = P2PView{};
    }
    if (g_p2p.own) {
        const cudaError_t e = cudaFree(g_p2p.own);
        if (e != cudaSuccess && rc == Q35CU_OK) rc = cuda_error(e, "cudaFree(p2p area)");
        g_p2p.own = nullptr;
        g_p2p.device = -1;
    }
    return rc;
}

Q35_API int q35cu_p2p_allreduce_f32(const float *in, float *out, size_t n, void *stream)
{
    if (!g_p2p.open) return set_error(Q35CU_ERR_NCCL, "p2p collectives not open");
    if (!in || !out || n > kP2PMaxElems) return set_error(Q35CU_ERR_ARG, "p2p_allreduce: n %zu (max %zu)", n, kP2PMaxElems);
    if (!n) return Q35CU_OK;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : default_stream();
    return launch_p2p(p2p_allreduce_kernel, chunks_for(n), st, in, out, (uint32_t)n);
}

Q35_API int q35cu_p2p_allgather_f32(const float *send, float *recv, size_t n_per_rank, void *stream)
{
    if (!g_p2p.open) return set_error(Q35CU_ERR_NCCL, "p2p collectives not open");
    if (!send || !recv || n_per_rank > kP2PMaxElems)
        return set_error(Q35CU_ERR_ARG, "p2p_allgather: n %zu (max %zu)", n_per_rank, kP2PMaxElems);
    if (!n_per_rank) return Q35CU_OK;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : default_stream();
    return launch_p2p(p2p_allgather_kernel, chunks_for(n_per_rank), st, send, recv, (uint32_t)n_per_rank);
}
