// Seeded synthetic FP8 weights generated in HBM, plus the small conversion
// kernels used at upload / download time.
//
// The generator follows the benchmark configurations' recipe: W0 ~ N(0,
// stddev^2) per element (counter-based: element g of stream `seed` always
// gets the same normal, whichever window or rank draws it), then per global
// 128x128 block s = bf16_rne(amax/448) and W = e4m3_rne(clamp(W0/s, +-448)),
// an all-zero block giving s = 0 and W = 0 -- the same block quantiser the
// engine applies to its in_proj_a/b tensors (qwen35-c/src/q35_model.c:327-343).
// The CPU oracle (oracle/q35_oracle.c, orc_synth_fp8) uses the same RNG.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "q35cu_internal.h"

namespace q35cu {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    // splitmix64 finaliser (Steele, Lea, Flood 2014)
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_normal(uint64_t seed, uint64_t g)
{
    const uint64_t h = mix64(seed * 0x9E3779B97F4A7C15ULL + (g + 1) * 0xD1B54A32D192ED03ULL);
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = (float)(uint32_t)((h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
}

__device__ __forceinline__ float bf16_round(float v)
{
    return __bfloat162float(__float2bfloat16_rn(v));
}

// One CTA per 128x128 block of the window; 256 threads, thread t owns row
// t/2 of the block and 64 consecutive columns.
__global__ void __launch_bounds__(256) synth_fp8_kernel(uint64_t seed, float stddev, uint32_t grows,
                                                        uint32_t gcols, uint32_t row0, uint32_t col0,
                                                        uint32_t nrows, uint32_t ncols, uint32_t bc,
                                                        uint8_t *W, float *S)
{
    __shared__ float wmax[8];
    const uint32_t bi = blockIdx.y, bj = blockIdx.x;
    const uint32_t lr = bi * 128 + (threadIdx.x >> 1);
    const uint32_t lc0 = bj * 128 + (threadIdx.x & 1) * 64;
    const uint32_t gr = row0 + lr;
    // amax over the GLOBAL block (a window never splits one, but its last
    // block may be cut by the window edge while the global block goes on)
    const uint32_t gbr0 = row0 + bi * 128, gbc0 = col0 + bj * 128;
    float v[64];
    float amax = 0.f;
    const bool row_in_global = gr < grows && gr < gbr0 + 128;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        const uint32_t gc = col0 + lc0 + j;
        v[j] = 0.f;
        if (row_in_global && gc < gcols && gc < gbc0 + 128) {
            v[j] = stddev * synth_normal(seed, (uint64_t)gr * gcols + gc);
            amax = fmaxf(amax, fabsf(v[j]));
        }
    }
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = wmax[0];
    for (int i = 1; i < 8; ++i) amax = fmaxf(amax, wmax[i]);
    const float s = bf16_round(amax / 448.0f);
    if (threadIdx.x == 0) S[(size_t)bi * bc + bj] = s;
    if (lr >= nrows) return;
    uint8_t *dst = W + (size_t)lr * ncols;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
        const uint32_t lc = lc0 + j;
        if (lc < ncols) {
            uint8_t b = 0;
            if (s != 0.f)
                b = (uint8_t)__nv_cvt_float_to_fp8(v[j] / s, __NV_SATFINITE, __NV_E4M3);
            dst[lc] = b;
        }
    }
}

__global__ void bf16_to_f32_kernel(const uint16_t *src, float *dst, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

__global__ void f32_to_bf16_kernel(const float *src, uint16_t *dst, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __bfloat16_as_ushort(__float2bfloat16_rn(src[i]));
}

__global__ void fill_nan_kernel(float *p, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = __int_as_float(0x7fc00000);
}

unsigned grid_for(size_t n)
{
    size_t b = (n + 255) / 256;
    const size_t cap = (size_t)device_sms() * 16;
    if (b > cap) b = cap;
    return (unsigned)(b ? b : 1);
}

}  // namespace

int launch_synth_fp8(uint64_t seed, float stddev, uint32_t grows, uint32_t gcols, uint32_t row0,
                     uint32_t col0, uint32_t nrows, uint32_t ncols, uint8_t *W, float *S,
                     cudaStream_t st)
{
    const uint32_t br = (nrows + 127) / 128, bc = (ncols + 127) / 128;
    if (br > 65535) return set_error(Q35CU_ERR_ARG, "synth: too many row blocks");
    synth_fp8_kernel<<<dim3(bc, br), 256, 0, st>>>(seed, stddev, grows, gcols, row0, col0, nrows,
                                                   ncols, bc, W, S);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

int launch_bf16_to_f32_scales(const uint16_t *src, float *dst, size_t n, cudaStream_t st)
{
    if (!n) return Q35CU_OK;
    bf16_to_f32_kernel<<<grid_for(n), 256, 0, st>>>(src, dst, n);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

int launch_f32_to_bf16_scales(const float *src, uint16_t *dst, size_t n, cudaStream_t st)
{
    if (!n) return Q35CU_OK;
    f32_to_bf16_kernel<<<grid_for(n), 256, 0, st>>>(src, dst, n);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

int launch_f32_to_bf16(const float *x, uint16_t *y, size_t n, cudaStream_t st)
{
    return launch_f32_to_bf16_scales(x, y, n, st);
}

int launch_fill_nan(float *p, size_t n, cudaStream_t st)
{
    if (!n) return Q35CU_OK;
    fill_nan_kernel<<<grid_for(n), 256, 0, st>>>(p, n);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    return Q35CU_OK;
}

}  // namespace q35cu
