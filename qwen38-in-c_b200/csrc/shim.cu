// libq35cuda host side: the reference-facing C-ABI (q35_mm.h) and the
// native API (q35cu.h).
//
// The q35_mm_* entry points keep the signatures and synchronous host-pointer
// semantics of qwen35-c/src/q35_mm.c:144-246.  Behind them:
//   * a residency cache keyed by (host W, host scale, rows, cols): the first
//     call uploads the weight (scales widened bf16 -> fp32, exact), later
//     calls reuse it -- the engine's weights are immutable mmaps
//     (qwen35-c/src/q35_model.c:253-273), so the key identifies the tensor;
//   * pinned host staging + one stream per device: copy x in, launch, copy
//     y out, synchronise, copy to the caller's buffer;
//   * errors: the signatures return void, so by default a failure aborts
//     with a message; Q35CU_ON_ERROR=record (or q35cu_set_error_mode) makes
//     it record the error and fill the outputs with NaN instead.
#include <dlfcn.h>
#include <nccl.h>  // types only: NCCL is resolved at run time (see load_nccl)

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "q35_mm.h"
#include "q35cu_internal.h"

#define Q35_API extern "C" __attribute__((visibility("default")))

// ------------------------------------------------------------------------
// errors
// ------------------------------------------------------------------------
namespace {
thread_local int t_err = Q35CU_OK;
thread_local char t_msg[512] = "";
std::atomic<int> g_mode{-1};
std::atomic<uint64_t> g_launches{0};

int error_mode()
{
    int m = g_mode.load();
    if (m < 0) {
        const char *e = getenv("Q35CU_ON_ERROR");
        m = (e && (!strcmp(e, "record") || !strcmp(e, "1"))) ? Q35CU_ON_ERROR_RECORD : Q35CU_ON_ERROR_ABORT;
        g_mode.store(m);
    }
    return m;
}
}  // namespace

namespace q35cu {

int set_error(int code, const char *fmt, ...)
{
    t_err = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof t_msg, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char *what)
{
    return set_error(e == cudaErrorMemoryAllocation ? Q35CU_ERR_NOMEM : Q35CU_ERR_CUDA, "%s: %s (%s)", what,
                     cudaGetErrorName(e), cudaGetErrorString(e));
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace q35cu

using namespace q35cu;

// ------------------------------------------------------------------------
// per-device state, budget, cache
// ------------------------------------------------------------------------
namespace {

struct DevState {
    bool ready = false;
    int sms = 0;
    int major = 0;
    cudaStream_t stream = nullptr;
    void *h_stage = nullptr;  // pinned, in + out
    size_t h_cap = 0;
    void *d_stage = nullptr;  // device, in + out
    size_t d_cap = 0;
    void *d_xbf = nullptr;    // GEMM workspace: prepared (f16) copy of a prefill activation batch
    size_t xbf_cap = 0;
    uint32_t *d_flag = nullptr;  // 4-byte scratch word for upload scans
    uint32_t *status_src[3] = {nullptr, nullptr, nullptr};  // the status words (host_call)
    void *h_stage_dev = nullptr;  // the device's view of h_stage (host-mapped)
    // completion signal of host-pointer decode calls (host_call_signal)
    uint32_t *sig_count = nullptr;  // device: CTAs out of the current launch
    uint32_t *sig_flag = nullptr;   // host-mapped: {seq, device status}
    uint32_t *sig_flag_dev = nullptr;
    uint32_t sig_seq = 0;
};

struct Key {
    const void *w, *s;
    uint32_t rows, cols;
    int kind;
    bool operator==(const Key &o) const
    {
        return w == o.w && s == o.s && rows == o.rows && cols == o.cols && kind == o.kind;
    }
};
struct KeyHash {
    size_t operator()(const Key &k) const
    {
        size_t h = std::hash<const void *>()(k.w);
        h ^= std::hash<const void *>()(k.s) + 0x9e3779b97f4a7c15ULL + (h << 6) + (h >> 2);
        h ^= ((size_t)k.rows << 32 | k.cols) + 0x9e3779b97f4a7c15ULL + (h << 6) + (h >> 2);
        return h ^ (size_t)k.kind;
    }
};
struct Entry {
    q35cu_weight *w;
    bool owned;    // false for q35cu_weight_bind
    uint64_t fp;   // content fingerprint of the host tensor at upload
};

std::recursive_mutex g_mu;
int g_device = 0;
std::vector<DevState> g_dev;
std::unordered_map<Key, Entry, KeyHash> g_cache;
size_t g_cache_bytes = 0;
size_t g_budget = 0;
size_t g_alloc_bytes = 0;

DevState *dev_state()
{
    if (g_dev.empty()) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            set_error(Q35CU_ERR_NODEV, "no CUDA device visible");
            return nullptr;
        }
        g_dev.resize(n);
    }
    if (g_device < 0 || g_device >= (int)g_dev.size()) {
        set_error(Q35CU_ERR_NODEV, "device %d out of range", g_device);
        return nullptr;
    }
    DevState &d = g_dev[g_device];
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != g_device) {
        if (cudaSetDevice(g_device) != cudaSuccess) {
            cuda_error(cudaGetLastError(), "cudaSetDevice");
            return nullptr;
        }
    }
    if (!d.ready) {
        cudaDeviceProp p;
        cudaError_t e = cudaGetDeviceProperties(&p, g_device);
        if (e != cudaSuccess) { cuda_error(e, "cudaGetDeviceProperties"); return nullptr; }
        if (p.major != 10) {
            set_error(Q35CU_ERR_NODEV, "device %d is sm_%d%d; this library is built for sm_100a only", g_device,
                      p.major, p.minor);
            return nullptr;
        }
        d.sms = p.multiProcessorCount;
        d.major = p.major;
        e = cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) { cuda_error(e, "cudaStreamCreate"); return nullptr; }
        e = cudaMalloc(reinterpret_cast<void **>(&d.d_flag), 16);
        if (e != cudaSuccess) { cuda_error(e, "cudaMalloc(flag)"); return nullptr; }
        d.ready = true;
    }
    return &d;
}

int ensure_stage(DevState *d, size_t bytes)
{
    bytes = (bytes + 255) & ~(size_t)255;
    if (bytes > d->h_cap) {
        if (d->h_stage) cudaFreeHost(d->h_stage);
        d->h_stage = nullptr;
        d->h_cap = 0;
        size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
        // mapped: the decode calls' kernels read their input from it and
        // write their output into it (host_call_signal)
        Q35CU_CUDA(cudaHostAlloc(&d->h_stage, cap, cudaHostAllocMapped));
        d->h_cap = cap;
        Q35CU_CUDA(cudaHostGetDevicePointer(&d->h_stage_dev, d->h_stage, 0));
    }
    if (bytes > d->d_cap) {
        if (d->d_stage) dev_free(d->d_stage, d->d_cap);
        d->d_stage = nullptr;
        d->d_cap = 0;
        size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
        int rc = dev_alloc(&d->d_stage, cap);
        if (rc) return rc;
        d->d_cap = cap;
    }
    return Q35CU_OK;
}

void weight_release(q35cu_weight *w)
{
    if (!w) return;
    int cur = 0;
    cudaGetDevice(&cur);
    if (w->device != cur) cudaSetDevice(w->device);
    dev_free(w->d_w, w->bytes - (w->d_s ? (size_t)w->rows_blk * w->cols_blk * 4 : 0));
    if (w->d_s) dev_free(w->d_s, (size_t)w->rows_blk * w->cols_blk * 4);
    if (w->device != cur) cudaSetDevice(cur);
    delete w;
}

// fail according to the error mode: abort, or record + NaN-fill host outputs
void fail_host(float *const *outs, const size_t *counts, int nout)
{
    if (error_mode() == Q35CU_ON_ERROR_ABORT) {
        fprintf(stderr, "libq35cuda: fatal: %s (code %d)\n", t_msg, t_err);
        abort();
    }
    for (int i = 0; i < nout; ++i)
        if (outs[i])
            for (size_t j = 0; j < counts[i]; ++j) outs[i][j] = __builtin_nanf("");
}

}  // namespace

namespace q35cu {

int device_sms()
{
    if (g_device >= 0 && g_device < (int)g_dev.size() && g_dev[g_device].ready) return g_dev[g_device].sms;
    DevState *d = dev_state();
    return d ? d->sms : 148;
}

cudaStream_t default_stream()
{
    if (g_device >= 0 && g_device < (int)g_dev.size() && g_dev[g_device].ready) return g_dev[g_device].stream;
    DevState *d = dev_state();
    return d ? d->stream : nullptr;
}

int dev_alloc(void **p, size_t bytes)
{
    *p = nullptr;
    if (g_budget && g_alloc_bytes + bytes > g_budget)
        return set_error(Q35CU_ERR_NOMEM, "device budget exceeded: %zu + %zu > %zu bytes", g_alloc_bytes, bytes,
                         g_budget);
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        return cuda_error(e, "cudaMalloc");
    }
    g_alloc_bytes += bytes;
    return Q35CU_OK;
}

void dev_free(void *p, size_t bytes)
{
    if (!p) return;
    cudaFree(p);
    g_alloc_bytes -= bytes < g_alloc_bytes ? bytes : g_alloc_bytes;
}

}  // namespace q35cu

// ------------------------------------------------------------------------
// weights
// ------------------------------------------------------------------------
namespace {

int weight_alloc(int kind, uint32_t rows, uint32_t cols, q35cu_weight **out)
{
    *out = nullptr;
    if (!rows || !cols) return set_error(Q35CU_ERR_ARG, "weight shape %ux%u", rows, cols);
    if (!dev_state()) return t_err;
    auto *w = new q35cu_weight{};
    w->kind = kind;
    w->rows = rows;
    w->cols = cols;
    w->rows_blk = (rows + 127) / 128;
    w->cols_blk = (cols + 127) / 128;
    w->device = g_device;
    const size_t wb = (size_t)rows * cols * (kind == 0 ? 1 : 2);
    int rc = dev_alloc(&w->d_w, wb);
    if (rc) { delete w; return rc; }
    w->bytes = wb;
    if (kind == 0) {
        const size_t sb = (size_t)w->rows_blk * w->cols_blk * 4;
        rc = dev_alloc(reinterpret_cast<void **>(&w->d_s), sb);
        if (rc) { dev_free(w->d_w, wb); delete w; return rc; }
        w->bytes += sb;
    }
    *out = w;
    return Q35CU_OK;
}

// copy host FP8 window + bf16 scale window into w (synchronous)
int weight_fill_fp8(q35cu_weight *w, const uint8_t *W, const uint16_t *sc, uint32_t cols, uint32_t row0,
                    uint32_t col0)
{
    DevState *d = dev_state();
    if (!d) return t_err;
    cudaStream_t st = d->stream;
    if (col0 == 0 && w->cols == cols) {
        Q35CU_CUDA(cudaMemcpyAsync(w->d_w, W + (size_t)row0 * cols, (size_t)w->rows * cols,
                                   cudaMemcpyHostToDevice, st));
    } else {
        Q35CU_CUDA(cudaMemcpy2DAsync(w->d_w, w->cols, W + (size_t)row0 * cols + col0, cols, w->cols, w->rows,
                                     cudaMemcpyHostToDevice, st));
    }
    const uint32_t gcb = (cols + 127) / 128;
    const size_t n = (size_t)w->rows_blk * w->cols_blk;
    int rc = ensure_stage(d, n * 2);
    if (rc) return rc;
    uint16_t *hs = static_cast<uint16_t *>(d->h_stage);
    Q35CU_CUDA(cudaStreamSynchronize(st));  // staging may be in use
    for (uint32_t i = 0; i < w->rows_blk; ++i)
        memcpy(hs + (size_t)i * w->cols_blk, sc + (size_t)(row0 / 128 + i) * gcb + col0 / 128,
               (size_t)w->cols_blk * 2);
    Q35CU_CUDA(cudaMemcpyAsync(d->d_stage, hs, n * 2, cudaMemcpyHostToDevice, st));
    rc = launch_bf16_to_f32_scales(static_cast<uint16_t *>(d->d_stage), w->d_s, n, st);
    if (rc) return rc;
    bool nan = false;
    rc = scan_nan_codes(static_cast<const uint8_t *>(w->d_w), (size_t)w->rows * w->cols, d->d_flag, st, &nan);
    if (rc) return rc;
    w->has_nan = nan;
    return Q35CU_OK;
}

// Content fingerprint of a host weight: 64 evenly spaced 8-byte words of
// the scale grid (all of it when smaller) and 8 of W, hashed in four
// independent lanes.  A cache hit whose fingerprint differs (the caller
// freed the tensor and reused the address for another one, whose scales
// differ almost everywhere) is treated as a miss.  It runs on every host
// call, so it reads few bytes: hashing a whole 11 KB scale grid took ~3 us
// a call.  Q35CU_CACHE_CHECK=0 skips the check.
uint64_t fingerprint(const void *W, size_t wbytes, const void *S, size_t sbytes)
{
    uint64_t h[4] = {0x9E3779B97F4A7C15ULL ^ wbytes, 0xC2B2AE3D27D4EB4FULL ^ sbytes, 0x165667B19E3779F9ULL,
                     0x27D4EB2F165667C5ULL};
    auto mix = [](uint64_t &x, uint64_t v) {
        x ^= v;
        x *= 0xFF51AFD7ED558CCDULL;
        x ^= x >> 32;
    };
    auto word = [](const uint8_t *base, size_t bytes, size_t off) {
        uint64_t v = 0;
        memcpy(&v, base + off, bytes - off < 8 ? bytes - off : 8);
        return v;
    };
    const uint8_t *sp = static_cast<const uint8_t *>(S);
    if (sbytes) {
        const size_t nw = (sbytes + 7) / 8, take = nw < 64 ? nw : 64;
        for (size_t j = 0; j < take; ++j) {
            const size_t wi = take == nw ? j : (nw - 1) * j / (take - 1);
            mix(h[j & 3], word(sp, sbytes, wi * 8));
        }
    }
    const uint8_t *wp = static_cast<const uint8_t *>(W);
    if (wbytes) {
        for (int j = 0; j < 8; ++j) {
            const size_t off = wbytes <= 8 ? 0 : ((wbytes - 8) * j / 7) & ~(size_t)7;
            mix(h[j & 3], word(wp, wbytes, off));
        }
    }
    uint64_t r = h[0];
    for (int i = 1; i < 4; ++i) mix(r, h[i]);
    return r;
}

bool cache_check_enabled()
{
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("Q35CU_CACHE_CHECK");
        on = !(e && !strcmp(e, "0"));
    }
    return on != 0;
}

// find or upload the weight for a host key (q35_mm_* path)
q35cu_weight *cached_weight(int kind, const void *W, const void *sc, uint32_t rows, uint32_t cols)
{
    Key k{W, sc, rows, cols, kind};
    const size_t wbytes = (size_t)rows * cols * (kind == 0 ? 1 : 2);
    const size_t sbytes = kind == 0 ? (size_t)((rows + 127) / 128) * ((cols + 127) / 128) * 2 : 0;
    const bool verify = cache_check_enabled();
    auto it = g_cache.find(k);
    // a bound entry's host key need not hold the tensor (q35cu_weight_bind): never read it
    if (it != g_cache.end() && !it->second.owned) return it->second.w;
    const uint64_t fp = verify ? fingerprint(W, wbytes, sc, sbytes) : 0;
    if (it != g_cache.end()) {
        if (!verify || it->second.fp == fp) return it->second.w;
        g_cache_bytes -= it->second.w->bytes;  // stale: same address, other contents
        weight_release(it->second.w);
        g_cache.erase(it);
    }
    q35cu_weight *w = nullptr;
    if (weight_alloc(kind, rows, cols, &w)) return nullptr;
    int rc;
    if (kind == 0) {
        rc = weight_fill_fp8(w, static_cast<const uint8_t *>(W), static_cast<const uint16_t *>(sc), cols, 0, 0);
    } else {
        DevState *d = dev_state();
        rc = cudaMemcpyAsync(w->d_w, W, (size_t)rows * cols * 2, cudaMemcpyHostToDevice, d->stream) == cudaSuccess
                 ? cudaStreamSynchronize(d->stream) == cudaSuccess ? Q35CU_OK : cuda_error(cudaGetLastError(), "sync")
                 : cuda_error(cudaGetLastError(), "cudaMemcpyAsync");
    }
    if (rc) { weight_release(w); return nullptr; }
    g_cache.emplace(k, Entry{w, true, fp});
    g_cache_bytes += w->bytes;
    return w;
}

GemvSeg seg_of(const q35cu_weight *w, float *Y, uint32_t ldy)
{
    GemvSeg g{};
    g.W = static_cast<const uint8_t *>(w->d_w);
    g.S = w->d_s;
    g.Y = Y;
    g.rows = w->rows;
    g.ldy = ldy;
    g.has_nan = w->has_nan;
    return g;
}

}  // namespace

// ------------------------------------------------------------------------
// q35cu.h: errors, device, cache
// ------------------------------------------------------------------------
Q35_API int q35cu_last_error(void) { return t_err; }
Q35_API const char *q35cu_last_error_message(void) { return t_msg; }
Q35_API void q35cu_clear_error(void) { t_err = Q35CU_OK; t_msg[0] = 0; }
Q35_API void q35cu_set_error_mode(int mode) { g_mode.store(mode ? Q35CU_ON_ERROR_RECORD : Q35CU_ON_ERROR_ABORT); }
Q35_API int q35cu_get_error_mode(void) { return error_mode(); }

Q35_API int q35cu_device_count(void)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

Q35_API int q35cu_set_device(int device)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    int n = q35cu_device_count();
    if (device < 0 || device >= n) return set_error(Q35CU_ERR_NODEV, "device %d of %d", device, n);
    g_device = device;
    return dev_state() ? Q35CU_OK : t_err;
}

Q35_API int q35cu_sm_count(void)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    DevState *d = dev_state();
    return d ? d->sms : 0;
}

Q35_API size_t q35cu_cache_bytes(void)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    return g_cache_bytes;
}

Q35_API void q35cu_set_memory_budget(size_t bytes)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    g_budget = bytes;
}

Q35_API void q35cu_release_all(void)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    for (auto &kv : g_cache)
        if (kv.second.owned) weight_release(kv.second.w);
    g_cache.clear();
    g_cache_bytes = 0;
}

Q35_API int q35cu_forget(const void *W)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    int n = 0;
    for (auto it = g_cache.begin(); it != g_cache.end();) {
        if (it->first.w == W) {
            if (it->second.owned) {
                g_cache_bytes -= it->second.w->bytes;
                weight_release(it->second.w);
            }
            it = g_cache.erase(it);
            ++n;
        } else {
            ++it;
        }
    }
    return n;
}

// ------------------------------------------------------------------------
// q35cu.h: weights
// ------------------------------------------------------------------------
Q35_API int q35cu_weight_upload_fp8_window(const uint8_t *W, const uint16_t *sc, uint32_t rows, uint32_t cols,
                                           uint32_t row0, uint32_t nrows, uint32_t col0, uint32_t ncols,
                                           q35cu_weight **out)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!out) return set_error(Q35CU_ERR_ARG, "out is NULL");
    *out = nullptr;
    if (!W || !sc) return set_error(Q35CU_ERR_ARG, "weight or scale pointer is NULL");
    if ((row0 & 127) || (col0 & 127)) return set_error(Q35CU_ERR_ARG, "window origin (%u,%u) not 128-aligned", row0, col0);
    if (!nrows || !ncols || row0 + nrows > rows || col0 + ncols > cols)
        return set_error(Q35CU_ERR_ARG, "window [%u+%u, %u+%u] outside %ux%u", row0, nrows, col0, ncols, rows, cols);
    q35cu_weight *w = nullptr;
    int rc = weight_alloc(0, nrows, ncols, &w);
    if (rc) return rc;
    rc = weight_fill_fp8(w, W, sc, cols, row0, col0);
    if (rc) { weight_release(w); return rc; }
    *out = w;
    return Q35CU_OK;
}

Q35_API int q35cu_weight_upload_fp8(const uint8_t *W, const uint16_t *sc, uint32_t rows, uint32_t cols,
                                    q35cu_weight **out)
{
    return q35cu_weight_upload_fp8_window(W, sc, rows, cols, 0, rows, 0, cols, out);
}

Q35_API int q35cu_weight_upload_bf16(const uint16_t *W, uint32_t rows, uint32_t cols, q35cu_weight **out)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!out) return set_error(Q35CU_ERR_ARG, "out is NULL");
    *out = nullptr;
    if (!W) return set_error(Q35CU_ERR_ARG, "weight pointer is NULL");
    q35cu_weight *w = nullptr;
    int rc = weight_alloc(1, rows, cols, &w);
    if (rc) return rc;
    DevState *d = dev_state();
    cudaError_t e = cudaMemcpy(w->d_w, W, (size_t)rows * cols * 2, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { weight_release(w); return cuda_error(e, "cudaMemcpy"); }
    (void)d;
    *out = w;
    return Q35CU_OK;
}

Q35_API int q35cu_weight_synth_fp8(uint64_t seed, float stddev, uint32_t grows, uint32_t gcols, uint32_t row0,
                                   uint32_t nrows, uint32_t col0, uint32_t ncols, q35cu_weight **out)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!out) return set_error(Q35CU_ERR_ARG, "out is NULL");
    *out = nullptr;
    if ((row0 & 127) || (col0 & 127)) return set_error(Q35CU_ERR_ARG, "window origin not 128-aligned");
    if (!nrows || !ncols || row0 + nrows > grows || col0 + ncols > gcols)
        return set_error(Q35CU_ERR_ARG, "window outside the global matrix");
    q35cu_weight *w = nullptr;
    int rc = weight_alloc(0, nrows, ncols, &w);
    if (rc) return rc;
    DevState *d = dev_state();
    rc = launch_synth_fp8(seed, stddev, grows, gcols, row0, col0, nrows, ncols, static_cast<uint8_t *>(w->d_w),
                          w->d_s, d->stream);
    bool nan = false;
    if (!rc) rc = scan_nan_codes(static_cast<const uint8_t *>(w->d_w), (size_t)nrows * ncols, d->d_flag, d->stream, &nan);
    if (!rc) w->has_nan = nan;
    if (rc) { weight_release(w); return rc; }
    *out = w;
    return Q35CU_OK;
}

Q35_API int q35cu_weight_download_fp8(const q35cu_weight *w, uint8_t *W, uint16_t *sc)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!w || w->kind != 0 || !W || !sc) return set_error(Q35CU_ERR_ARG, "download: bad arguments");
    DevState *d = dev_state();
    if (!d) return t_err;
    Q35CU_CUDA(cudaMemcpy(W, w->d_w, (size_t)w->rows * w->cols, cudaMemcpyDeviceToHost));
    const size_t n = (size_t)w->rows_blk * w->cols_blk;
    int rc = ensure_stage(d, n * 2);
    if (rc) return rc;
    rc = launch_f32_to_bf16_scales(w->d_s, static_cast<uint16_t *>(d->d_stage), n, d->stream);
    if (rc) return rc;
    Q35CU_CUDA(cudaMemcpyAsync(sc, d->d_stage, n * 2, cudaMemcpyDeviceToHost, d->stream));
    Q35CU_CUDA(cudaStreamSynchronize(d->stream));
    return Q35CU_OK;
}

// ---- safetensors preload ---------------------------------------------------
//
// The engine maps every shard read-only and binds its matmul operands as
// pointers into the mappings (qwen35-c/src/q35_model.c:204-208, 252-273:
// tensor "X.weight" F8_E4M3 [rows, cols] with "X.weight_scale_inv" BF16
// [ceil(rows/128), ceil(cols/128)]; lm_head.weight BF16 for q35_mm_bf16).
// q35cu_preload_safetensors walks one mapped shard in file order and uploads
// those operands now, keyed by exactly those pointers, so the first forward
// pass finds them resident instead of uploading on first touch.  A weight and
// its scale may sit in different shards: the first one seen waits, by name,
// until the other's shard is preloaded.
namespace {

// A minimal JSON reader for the safetensors header: a flat object of
// name -> {"dtype": s, "shape": [n...], "data_offsets": [a, b]} (plus
// "__metadata__").  Unknown members are skipped.
struct JsonCursor {
    const char *p, *e;
    bool ok = true;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool eat(char c)
    {
        ws();
        if (p < e && *p == c) { ++p; return true; }
        return false;
    }
    bool str(std::string *out)
    {
        ws();
        if (p >= e || *p != '"') return ok = false;
        ++p;
        std::string v;
        while (p < e && *p != '"') {
            if (*p == '\\') {
                if (++p >= e) return ok = false;
                const char c = *p;
                if (c == 'u') {  // names are ASCII in practice; keep the escape literally
                    v += "\\u";
                } else {
                    v += c == 'n' ? '\n' : c == 't' ? '\t' : c == 'r' ? '\r' : c == 'b' ? '\b' : c == 'f' ? '\f' : c;
                }
                ++p;
                continue;
            }
            v += *p++;
        }
        if (p >= e) return ok = false;
        ++p;
        if (out) *out = v;
        return true;
    }
    bool num(uint64_t *out)
    {
        ws();
        if (p >= e || *p < '0' || *p > '9') return ok = false;
        uint64_t v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            v = v * 10 + (uint64_t)(*p - '0');
            ++p;
        }
        if (out) *out = v;
        return true;
    }
    bool skip()  // any value
    {
        ws();
        if (p >= e) return ok = false;
        if (*p == '"') return str(nullptr);
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            ++p;
            if (eat(close)) return true;
            for (;;) {
                if (close == '}') {
                    if (!str(nullptr) || !eat(':')) return ok = false;
                }
                if (!skip()) return false;
                if (eat(close)) return true;
                if (!eat(',')) return ok = false;
            }
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;  // number, true, false, null
        return true;
    }
};

struct StTensor {
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t off0 = 0, off1 = 0;
};

// calls fn(name, tensor) for every tensor of the header; false if malformed
template <class F>
bool st_header(const uint8_t *base, size_t len, F &&fn)
{
    if (len < 8) return false;
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
    if (hlen > len - 8) return false;
    JsonCursor j{reinterpret_cast<const char *>(base + 8), reinterpret_cast<const char *>(base + 8 + hlen)};
    if (!j.eat('{')) return false;
    if (j.eat('}')) return true;
    for (;;) {
        std::string name;
        if (!j.str(&name) || !j.eat(':')) return false;
        if (name == "__metadata__") {
            if (!j.skip()) return false;
        } else {
            StTensor t;
            if (!j.eat('{')) return false;
            if (!j.eat('}')) {
                for (;;) {
                    std::string key;
                    if (!j.str(&key) || !j.eat(':')) return false;
                    if (key == "dtype") {
                        if (!j.str(&t.dtype)) return false;
                    } else if (key == "shape" || key == "data_offsets") {
                        if (!j.eat('[')) return false;
                        std::vector<uint64_t> v;
                        if (!j.eat(']')) {
                            for (;;) {
                                uint64_t x;
                                if (!j.num(&x)) return false;
                                v.push_back(x);
                                if (j.eat(']')) break;
                                if (!j.eat(',')) return false;
                            }
                        }
                        if (key == "shape") t.shape = v;
                        else if (v.size() == 2) { t.off0 = v[0]; t.off1 = v[1]; }
                        else return false;
                    } else if (!j.skip()) {
                        return false;
                    }
                    if (j.eat('}')) break;
                    if (!j.eat(',')) return false;
                }
            }
            if (t.off1 < t.off0 || t.off1 > len - 8 - hlen) return false;
            fn(name, t, base + 8 + hlen + t.off0);
        }
        if (j.eat('}')) return true;
        if (!j.eat(',')) return false;
    }
}

struct StHalf {
    const uint8_t *p;
    uint64_t d0, d1;  // shape
};
std::unordered_map<std::string, StHalf> g_st_w, g_st_s;  // unmatched FP8 weights / scale grids, by weight name
size_t g_preload_bytes = 0;

}  // namespace

Q35_API int q35cu_preload_safetensors(const void *base, size_t len)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!base) return set_error(Q35CU_ERR_ARG, "preload: NULL mapping");
    if (!dev_state()) return t_err;
    const uint8_t *b = static_cast<const uint8_t *>(base);
    static const std::string kSuffix = "_scale_inv";
    std::vector<std::pair<StHalf, StHalf>> pairs;  // (weight, scale) in file order
    std::vector<StHalf> bf16;                      // lm_head
    const bool parsed = st_header(b, len, [&](const std::string &name, const StTensor &t, const uint8_t *p) {
        if (t.shape.size() != 2) return;
        const StHalf h{p, t.shape[0], t.shape[1]};
        if (t.dtype == "F8_E4M3") {
            auto it = g_st_s.find(name);
            if (it != g_st_s.end()) { pairs.push_back({h, it->second}); g_st_s.erase(it); }
            else g_st_w[name] = h;
        } else if (t.dtype == "BF16" && name.size() > kSuffix.size() &&
                   name.compare(name.size() - kSuffix.size(), kSuffix.size(), kSuffix) == 0) {
            const std::string wname = name.substr(0, name.size() - kSuffix.size());
            auto it = g_st_w.find(wname);
            if (it != g_st_w.end()) { pairs.push_back({it->second, h}); g_st_w.erase(it); }
            else g_st_s[wname] = h;
        } else if (t.dtype == "BF16" && name == "lm_head.weight") {
            bf16.push_back(h);
        }
    });
    if (!parsed) return set_error(Q35CU_ERR_ARG, "preload: not a safetensors header");
    for (const auto &pr : pairs) {
        const StHalf &w = pr.first, &sc = pr.second;
        if (w.d0 > 0xFFFFFFFFull || w.d1 > 0xFFFFFFFFull || sc.d0 != (w.d0 + 127) / 128 || sc.d1 != (w.d1 + 127) / 128)
            continue;  // not a block-scaled pair the engine would bind
        if (!cached_weight(0, w.p, sc.p, (uint32_t)w.d0, (uint32_t)w.d1)) return t_err;
        g_preload_bytes += w.d0 * w.d1;
    }
    for (const auto &h : bf16) {
        if (h.d0 > 0xFFFFFFFFull || h.d1 > 0xFFFFFFFFull) continue;
        if (!cached_weight(1, h.p, nullptr, (uint32_t)h.d0, (uint32_t)h.d1)) return t_err;
        g_preload_bytes += h.d0 * h.d1 * 2;
    }
    return Q35CU_OK;
}

Q35_API void q35cu_preload_forget(const void *base, size_t len)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    const uint8_t *lo = static_cast<const uint8_t *>(base), *hi = lo + len;
    for (auto *m : {&g_st_w, &g_st_s})
        for (auto it = m->begin(); it != m->end();)
            it = (it->second.p >= lo && it->second.p < hi) ? m->erase(it) : std::next(it);
}

Q35_API size_t q35cu_preload_bytes(void)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    return g_preload_bytes;
}

Q35_API int q35cu_weight_bind(const uint8_t *host_W, const uint16_t *host_sc, const q35cu_weight *w)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!host_W || !host_sc || !w || w->kind != 0) return set_error(Q35CU_ERR_ARG, "bind: bad arguments");
    Key k{host_W, host_sc, w->rows, w->cols, 0};
    auto it = g_cache.find(k);
    if (it != g_cache.end()) {
        if (it->second.owned) {
            g_cache_bytes -= it->second.w->bytes;
            weight_release(it->second.w);
        }
        g_cache.erase(it);
    }
    g_cache.emplace(k, Entry{const_cast<q35cu_weight *>(w), false, 0});
    return Q35CU_OK;
}

Q35_API void q35cu_weight_free(q35cu_weight *w)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!w) return;
    for (auto it = g_cache.begin(); it != g_cache.end();) {
        if (it->second.w == w) {
            if (it->second.owned) g_cache_bytes -= w->bytes;
            it = g_cache.erase(it);
        } else {
            ++it;
        }
    }
    weight_release(w);
}

Q35_API uint32_t q35cu_weight_rows(const q35cu_weight *w) { return w ? w->rows : 0; }
Q35_API uint32_t q35cu_weight_cols(const q35cu_weight *w) { return w ? w->cols : 0; }
Q35_API size_t q35cu_weight_device_bytes(const q35cu_weight *w) { return w ? w->bytes : 0; }

// ------------------------------------------------------------------------
// q35cu.h: device-pointer compute
// ------------------------------------------------------------------------
static cudaStream_t pick(void *stream)
{
    return stream ? static_cast<cudaStream_t>(stream) : default_stream();
}

Q35_API int q35cu_gemv_fp8(const q35cu_weight *w, const float *X, uint32_t ldx, uint32_t m, float *Y, uint32_t ldy,
                           void *stream)
{
    if (!w || w->kind != 0 || !X || !Y) return set_error(Q35CU_ERR_ARG, "gemv_fp8: bad arguments");
    if (!m) return Q35CU_OK;
    if (ldx < w->cols || ldy < w->rows) return set_error(Q35CU_ERR_ARG, "gemv_fp8: ld smaller than the row");
    GemvSeg g = seg_of(w, Y, ldy);
    return launch_gemv(0, &g, 1, X, w->cols, ldx, m, pick(stream));
}

Q35_API int q35cu_multi_fp8(const q35cu_weight *const w[4], const float *X, uint32_t ldx, uint32_t m,
                            float *const Y[4], void *stream)
{
    if (!w || !Y || !X) return set_error(Q35CU_ERR_ARG, "multi_fp8: bad arguments");
    GemvSeg segs[4];
    int n = 0;
    uint32_t K = 0;
    for (int s = 0; s < 4; ++s) {
        if (!w[s]) continue;
        if (w[s]->kind != 0 || !Y[s]) return set_error(Q35CU_ERR_ARG, "multi_fp8: segment %d", s);
        if (K && w[s]->cols != K) return set_error(Q35CU_ERR_ARG, "multi_fp8: segments disagree on cols");
        K = w[s]->cols;
        segs[n++] = seg_of(w[s], Y[s], w[s]->rows);
    }
    if (!n || !m) return Q35CU_OK;
    if (ldx < K) return set_error(Q35CU_ERR_ARG, "multi_fp8: ldx < cols");
    return launch_gemv(0, segs, n, X, K, ldx, m, pick(stream));
}

Q35_API int q35cu_multi_fp8_tp(const q35cu_weight *const w[4], const float *X, float *const Y[4], int mode,
                               float *gathered, void *stream)
{
    if (!w || !Y || !X) return set_error(Q35CU_ERR_ARG, "multi_fp8_tp: bad arguments");
    if (mode != Q35CU_TP_ALLREDUCE && mode != Q35CU_TP_ALLGATHER)
        return set_error(Q35CU_ERR_ARG, "multi_fp8_tp: mode %d", mode);
    GemvSeg segs[4];
    int n = 0;
    uint32_t K = 0;
    for (int s = 0; s < 4; ++s) {
        if (!w[s]) continue;
        if (w[s]->kind != 0 || !Y[s]) return set_error(Q35CU_ERR_ARG, "multi_fp8_tp: segment %d", s);
        if (K && w[s]->cols != K) return set_error(Q35CU_ERR_ARG, "multi_fp8_tp: segments disagree on cols");
        K = w[s]->cols;
        segs[n++] = seg_of(w[s], Y[s], w[s]->rows);
    }
    if (!n) return Q35CU_OK;
    GemvTp tp;
    tp.mode = mode;
    tp.gathered = gathered;
    return launch_gemv(0, segs, n, X, K, K, 1, pick(stream), tp);
}

struct q35cu_chain {
    std::vector<uint8_t> ops;  // chain_op_bytes() per op
    uint32_t n = 0;
    void *d_ops = nullptr;
    size_t d_cap = 0;
    uint32_t *d_bar = nullptr;
    uint32_t layout[5] = {};
    bool dirty = true;
    int device = -1;
};

Q35_API int q35cu_chain_create(q35cu_chain **out)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!out) return set_error(Q35CU_ERR_ARG, "chain_create: NULL");
    *out = nullptr;
    if (!dev_state()) return t_err;
    q35cu_chain *c = new (std::nothrow) q35cu_chain;
    if (!c) return set_error(Q35CU_ERR_NOMEM, "chain_create");
    c->device = g_device;
    *out = c;
    return Q35CU_OK;
}

Q35_API int q35cu_chain_add(q35cu_chain *c, const q35cu_weight *const w[4], const float *X, float *const Y[4],
                            int mode, float *gathered)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!c || !w || !X || !Y) return set_error(Q35CU_ERR_ARG, "chain_add: bad arguments");
    if (mode != 0 && mode != Q35CU_TP_ALLREDUCE && mode != Q35CU_TP_ALLGATHER)
        return set_error(Q35CU_ERR_ARG, "chain_add: mode %d", mode);
    if (!dev_state()) return t_err;
    if (g_device != c->device) return set_error(Q35CU_ERR_ARG, "chain_add: chain belongs to device %d", c->device);
    GemvSeg segs[4];
    int n = 0;
    uint32_t K = 0;
    for (int s = 0; s < 4; ++s) {
        if (!w[s]) continue;
        if (w[s]->kind != 0 || !Y[s]) return set_error(Q35CU_ERR_ARG, "chain_add: segment %d", s);
        if (K && w[s]->cols != K) return set_error(Q35CU_ERR_ARG, "chain_add: segments disagree on cols");
        K = w[s]->cols;
        segs[n++] = seg_of(w[s], Y[s], w[s]->rows);
    }
    if (!n) return set_error(Q35CU_ERR_ARG, "chain_add: no weight");
    GemvTp tp;
    tp.mode = mode;
    tp.gathered = gathered;
    const size_t ob = chain_op_bytes();
    c->ops.resize((size_t)(c->n + 1) * ob);
    const int rc = chain_build_op(segs, n, X, K, tp, c->ops.data() + (size_t)c->n * ob);
    if (rc) {
        c->ops.resize((size_t)c->n * ob);
        return rc;
    }
    ++c->n;
    c->dirty = true;
    return Q35CU_OK;
}

Q35_API int q35cu_chain_run(q35cu_chain *c, void *stream)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!c) return set_error(Q35CU_ERR_ARG, "chain_run: NULL");
    if (!dev_state()) return t_err;
    if (g_device != c->device) return set_error(Q35CU_ERR_ARG, "chain_run: chain belongs to device %d", c->device);
    if (!c->n) return Q35CU_OK;
    if (c->dirty) {  // lay out and upload the op table (synchronous: not inside a stream capture)
        int rc = chain_layout(c->ops.data(), c->n, c->layout);
        if (rc) return rc;
        if (c->ops.size() > c->d_cap) {
            if (c->d_ops) dev_free(c->d_ops, c->d_cap);
            c->d_ops = nullptr;
            c->d_cap = 0;
            rc = dev_alloc(&c->d_ops, c->ops.size());
            if (rc) return rc;
            c->d_cap = c->ops.size();
        }
        if (!c->d_bar) {
            void *p = nullptr;
            rc = dev_alloc(&p, 256);
            if (rc) return rc;
            c->d_bar = static_cast<uint32_t *>(p);
            Q35CU_CUDA(cudaMemset(c->d_bar, 0, 256));
        }
        Q35CU_CUDA(cudaMemcpy(c->d_ops, c->ops.data(), c->ops.size(), cudaMemcpyHostToDevice));
        c->dirty = false;
    }
    return launch_chain(c->d_ops, c->n, c->d_bar, c->layout, pick(stream));
}

Q35_API void q35cu_chain_free(q35cu_chain *c)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!c) return;
    if (c->d_ops) dev_free(c->d_ops, c->d_cap);
    if (c->d_bar) dev_free(c->d_bar, 256);
    delete c;
}

Q35_API int q35cu_gemv_fp8_tp(const q35cu_weight *w, const float *X, float *Y, int mode, float *gathered,
                              void *stream)
{
    const q35cu_weight *ws[4] = {w, nullptr, nullptr, nullptr};
    float *ys[4] = {Y, nullptr, nullptr, nullptr};
    if (!w) return set_error(Q35CU_ERR_ARG, "gemv_fp8_tp: bad arguments");
    return q35cu_multi_fp8_tp(ws, X, ys, mode, gathered, stream);
}

Q35_API size_t q35cu_gemv_fp8_tc_workspace_bytes(uint32_t m, uint32_t cols)
{
    return gemm_exact_workspace_bytes(m, cols);
}

Q35_API int q35cu_gemv_fp8_tc(const q35cu_weight *w, const float *X, uint32_t m, float *Y, void *workspace,
                              size_t workspace_bytes, void *stream)
{
    if (!w || w->kind != 0 || !X || !Y) return set_error(Q35CU_ERR_ARG, "gemv_fp8_tc: bad arguments");
    if (!m) return Q35CU_OK;
    const size_t need = gemm_exact_workspace_bytes(m, w->cols);
    if (!workspace || workspace_bytes < need)
        return set_error(Q35CU_ERR_ARG, "gemv_fp8_tc: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    return launch_gemm_exact(w, X, m, Y, workspace, pick(stream));
}

Q35_API size_t q35cu_gemm_fp8_workspace_bytes(uint32_t m, uint32_t cols)
{
    return gemm_workspace_bytes(m, cols);
}

Q35_API int q35cu_gemm_fp8(const q35cu_weight *w, const uint16_t *Xb, uint32_t m, float *Y, void *workspace,
                           size_t workspace_bytes, void *stream)
{
    if (!w || w->kind != 0 || !Xb || !Y) return set_error(Q35CU_ERR_ARG, "gemm_fp8: bad arguments");
    if (!m) return Q35CU_OK;
    const size_t need = gemm_workspace_bytes(m, w->cols);
    if (!workspace || workspace_bytes < need)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    return launch_gemm_bf16(w, Xb, false, m, Y, workspace, pick(stream));
}

Q35_API int q35cu_gemm_fp8_f32(const q35cu_weight *w, const float *X, uint32_t m, float *Y, void *workspace,
                               size_t workspace_bytes, void *stream)
{
    if (!w || w->kind != 0 || !X || !Y) return set_error(Q35CU_ERR_ARG, "gemm_fp8_f32: bad arguments");
    if (!m) return Q35CU_OK;
    const size_t need = gemm_workspace_bytes(m, w->cols);
    if (!workspace || workspace_bytes < need)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8_f32: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    return launch_gemm_bf16(w, X, true, m, Y, workspace, pick(stream));
}

Q35_API int q35cu_gemm_fp8_multi(const q35cu_weight *const *w, uint32_t nw, const void *X, int x_f32, uint32_t m,
                                 float *const *Y, void *workspace, size_t workspace_bytes, void *stream)
{
    if (!w || !X || !Y || nw < 1 || nw > 4) return set_error(Q35CU_ERR_ARG, "gemm_fp8_multi: bad arguments");
    for (uint32_t i = 0; i < nw; ++i) {
        if (!w[i] || w[i]->kind != 0 || !Y[i]) return set_error(Q35CU_ERR_ARG, "gemm_fp8_multi: bad weight or output %u", i);
        if (w[i]->cols != w[0]->cols)
            return set_error(Q35CU_ERR_ARG, "gemm_fp8_multi: weight %u has %u columns, weight 0 %u", i, w[i]->cols,
                             w[0]->cols);
    }
    if (!m) return Q35CU_OK;
    const size_t need = gemm_workspace_bytes(m, w[0]->cols);
    if (!workspace || workspace_bytes < need)
        return set_error(Q35CU_ERR_ARG, "gemm_fp8_multi: workspace of %zu bytes, %zu needed", workspace_bytes, need);
    return launch_gemm_bf16_multi(w, Y, nw, X, x_f32 != 0, m, workspace, pick(stream));
}

Q35_API int q35cu_gemm_reserve_sms(int n) { return gemm_reserve_sms(n); }

Q35_API int q35cu_f32_to_bf16(const float *x, uint16_t *y, size_t n, void *stream)
{
    if (!x || !y) return set_error(Q35CU_ERR_ARG, "f32_to_bf16: NULL");
    return launch_f32_to_bf16(x, y, n, pick(stream));
}

Q35_API int q35cu_swiglu(const float *g, const float *u, float *o, size_t n, void *stream)
{
    if (!g || !u || !o) return set_error(Q35CU_ERR_ARG, "swiglu: NULL");
    return launch_swiglu(g, u, o, n, pick(stream));
}

Q35_API int q35cu_gemv_bf16(const q35cu_weight *w, const float *x, float *y, void *stream)
{
    if (!w || w->kind != 1 || !x || !y) return set_error(Q35CU_ERR_ARG, "gemv_bf16: bad arguments");
    GemvSeg g = seg_of(w, y, w->rows);
    return launch_gemv(1, &g, 1, x, w->cols, w->cols, 1, pick(stream));
}

Q35_API const char *q35cu_build_info(void)
{
    return "libq35cuda sm_100a (nvcc " Q35CU_STR(__CUDACC_VER_MAJOR__) "." Q35CU_STR(__CUDACC_VER_MINOR__) ")";
}

Q35_API uint64_t q35cu_launch_count(void) { return g_launches.load(); }

Q35_API int q35cu_device_status(uint32_t *status, int clear)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!status) return set_error(Q35CU_ERR_ARG, "status is NULL");
    if (!dev_state()) return t_err;
    return device_status(status, clear != 0);
}

Q35_API int q35cu_gemm_timeout_info(uint32_t out[4])
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!out) return set_error(Q35CU_ERR_ARG, "out is NULL");
    if (!dev_state()) return t_err;
    return gemm_timeout_info(out);
}

// ------------------------------------------------------------------------
// q35_mm.h: the reference-facing entry points
// ------------------------------------------------------------------------
__attribute__((visibility("default"))) float q35_mm_fp8_lut[256];
namespace {
std::once_flag g_lut_once;
}

Q35_API float q35_mm_e4m3_to_f32(uint8_t v)
{
    const int neg = v >> 7, e = (v >> 3) & 15, m = v & 7;
    float mag;
    if (e == 15 && m == 7) return __builtin_nanf("");
    if (e == 0) mag = (float)m * (1.0f / 512.0f);
    else mag = ldexpf((float)(8 + m), e - 10);
    return neg ? -mag : mag;
}

Q35_API float q35_mm_bf16_to_f32(uint16_t v)
{
    uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

Q35_API void q35_mm_init(void)
{
    std::call_once(g_lut_once, [] {
        for (int i = 0; i < 256; ++i) q35_mm_fp8_lut[i] = q35_mm_e4m3_to_f32((uint8_t)i);
    });
}

Q35_API const char *q35_mm_impl_fp8(void) { return "sm_100a"; }

namespace {

// batches of at least this many tokens take the tensor-core GEMM
// (Q35CU_GEMM_MIN_TOKENS overrides; the default keeps M <= 64 on the fp32 GEMV)
uint32_t gemm_min_tokens()
{
    static uint32_t v = 0;
    if (!v) {
        const char *e = getenv("Q35CU_GEMM_MIN_TOKENS");
        v = (e && atoi(e) > 0) ? (uint32_t)atoi(e) : 128u;
    }
    return v;
}

// batches of at least this many (and fewer than gemm_min_tokens) tokens take
// the tensor cores with exact fp32 activations (hi/lo split); smaller ones
// stay on the decode GEMV, bit-identical to single calls
// (Q35CU_GEMV_TC_MIN_TOKENS overrides; 0 disables)
uint32_t gemv_tc_min_tokens()
{
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("Q35CU_GEMV_TC_MIN_TOKENS");
        v = e ? atoi(e) : 16;
        if (v <= 0) v = 0x7FFFFFFF;
    }
    return (uint32_t)v;
}

// the three status words, side by side (for host_call's single copy back)
__global__ void gather_status_kernel(const uint32_t *a, const uint32_t *b, const uint32_t *c, uint32_t *dst)
{
    if (threadIdx.x == 0) {
        dst[0] = *reinterpret_cast<const volatile uint32_t *>(a);
        dst[1] = *reinterpret_cast<const volatile uint32_t *>(b);
        dst[2] = *reinterpret_cast<const volatile uint32_t *>(c);
        dst[3] = 0;
    }
}

// a bounded device-side wait that gave up leaves a code in the status word
int check_device_status()
{
    uint32_t g = 0, where[4] = {0, 0, 0, 0};
    int rc = gemm_status(&g, false);
    if (!rc && g) rc = gemm_timeout_info(where);
    if (rc) return rc;
    uint32_t st = 0;
    rc = device_status(&st, true);
    if (rc) return rc;
    if (g)
        return set_error((int)g, "a tensor-core GEMM wait gave up (status %u; role %u, CTA %u, block %u, thread %u)",
                         g, where[0], where[1], where[2], where[3]);
    if (st) return set_error((int)st, "a device-side wait gave up (status %u)", st);
    return Q35CU_OK;
}

// stage X in, run `fn` (which launches on d->stream into the device output
// region), stage the output back and hand the host copy to `deliver` (which
// copies it into the caller's buffers).  in_bytes / out_bytes are exact byte
// counts.  The three device status words travel back behind the output in
// the same copy (one tiny kernel gathers them), so a call costs one H2D, one
// D2H and one synchronisation; they are read again (and cleared) only when
// one is set.
template <class F, class G>
int host_call_ex(const void *X, size_t in_bytes, size_t out_bytes, F &&fn, G &&deliver)
{
    DevState *d = dev_state();
    if (!d) return t_err;
    if (!d->status_src[0]) {
        d->status_src[0] = device_status_word();
        d->status_src[1] = gemm_status_word();
        d->status_src[2] = p2p_status_word();
        if (!d->status_src[0] || !d->status_src[1] || !d->status_src[2])
            return set_error(Q35CU_ERR_CUDA, "status words not found");
    }
    const size_t in_al = (in_bytes + 255) & ~(size_t)255;
    const size_t out_al = (out_bytes + 15) & ~(size_t)15;
    int rc = ensure_stage(d, in_al + out_al + 16);
    if (rc) return rc;
    char *h = static_cast<char *>(d->h_stage);
    char *dv = static_cast<char *>(d->d_stage);
    memcpy(h, X, in_bytes);
    Q35CU_CUDA(cudaMemcpyAsync(dv, h, in_bytes, cudaMemcpyHostToDevice, d->stream));
    rc = fn(reinterpret_cast<const float *>(dv), reinterpret_cast<float *>(dv + in_al), d->stream);
    if (rc) return rc;
    uint32_t *st_dev = reinterpret_cast<uint32_t *>(dv + in_al + out_al);
    gather_status_kernel<<<1, 32, 0, d->stream>>>(d->status_src[0], d->status_src[1], d->status_src[2], st_dev);
    count_launch();
    Q35CU_CUDA(cudaGetLastError());
    Q35CU_CUDA(cudaMemcpyAsync(h + in_al, dv + in_al, out_al + 16, cudaMemcpyDeviceToHost, d->stream));
    Q35CU_CUDA(cudaStreamSynchronize(d->stream));
    const uint32_t *st = reinterpret_cast<const uint32_t *>(h + in_al + out_al);
    if (st[0] | st[1] | st[2]) {
        rc = check_device_status();  // reads and clears all three
        if (rc) return rc;
    }
    deliver(static_cast<const char *>(h + in_al));
    return Q35CU_OK;
}

template <class F>
int host_call(const void *X, size_t in_bytes, void *Y, size_t out_bytes, F &&fn)
{
    return host_call_ex(X, in_bytes, out_bytes, fn, [&](const char *out) { memcpy(Y, out, out_bytes); });
}

// The decode calls (q35_mm_fp8, q35_mm_fp8_multi4, small q35_mm_fp8_batch)
// on a latency budget.  Each is a synchronous round trip, so per call the
// fixed costs count as much as the kernel: on a B200 host a DMA copy in, a
// status-gather kernel, a DMA copy out and a stream synchronisation measured
// ~20 us beyond the kernel's own launch and run.  Here instead
//   * the input is copied in by one DMA from the pinned staging buffer (a
//     one-CTA copy kernel reading the mapped buffer instead measured slower);
//   * the GEMV writes its outputs straight into the mapped staging buffer;
//   * its last CTA writes {sequence number, device status word} into a
//     host-mapped flag after every output is visible, and this thread polls
//     the flag instead of synchronising the stream.
// A flag that does not arrive within kSignalWaitS seconds ends the wait with
// the stream's error, or Q35CU_ERR_TIMEOUT.
constexpr size_t kSignalOutMax = 4 << 20;
constexpr double kSignalWaitS = 60.0;

double wall_s()
{
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

template <class F, class G>
int host_call_signal(const void *X, size_t in_bytes, size_t out_bytes, F &&launch, G &&deliver)
{
    DevState *d = dev_state();
    if (!d) return t_err;
    if (!d->sig_count) {
        void *c = nullptr;
        int rc = dev_alloc(&c, 256);
        if (rc) return rc;
        Q35CU_CUDA(cudaMemset(c, 0, 256));
        void *f = nullptr;
        Q35CU_CUDA(cudaHostAlloc(&f, 64, cudaHostAllocMapped));
        memset(f, 0, 64);
        Q35CU_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void **>(&d->sig_flag_dev), f, 0));
        d->sig_flag = static_cast<uint32_t *>(f);
        d->sig_count = static_cast<uint32_t *>(c);
    }
    const size_t in_al = (in_bytes + 255) & ~(size_t)255;
    const size_t out_al = (out_bytes + 255) & ~(size_t)255;
    int rc = ensure_stage(d, in_al + out_al);
    if (rc) return rc;
    char *h = static_cast<char *>(d->h_stage);
    char *hdev = static_cast<char *>(d->h_stage_dev);
    char *dv = static_cast<char *>(d->d_stage);
    memcpy(h, X, in_bytes);
    Q35CU_CUDA(cudaMemcpyAsync(dv, h, in_bytes, cudaMemcpyHostToDevice, d->stream));
    HostSignal sig;
    sig.count = d->sig_count;
    sig.flag = d->sig_flag_dev;
    sig.seq = ++d->sig_seq;
    if (sig.seq == 0) sig.seq = ++d->sig_seq;  // 0 is the flag's initial value
    rc = launch(reinterpret_cast<const float *>(dv), reinterpret_cast<float *>(hdev + in_al), d->stream, &sig);
    if (rc) return rc;
    volatile uint32_t *flag = d->sig_flag;
    const double t0 = wall_s();
    for (uint32_t i = 1; flag[0] != sig.seq; ++i) {
#if defined(__x86_64__)
        __builtin_ia32_pause();
#endif
        if ((i & 4095) == 0 && wall_s() - t0 > kSignalWaitS) {
            Q35CU_CUDA(cudaStreamSynchronize(d->stream));
            if (flag[0] == sig.seq) break;
            return set_error(Q35CU_ERR_TIMEOUT, "decode call: completion signal not seen after %.0f s", kSignalWaitS);
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    if (flag[1]) {
        rc = check_device_status();  // reads and clears the status words
        if (rc) return rc;
    }
    deliver(static_cast<const char *>(h + in_al));
    return Q35CU_OK;
}

// the decode GEMV with a completion signal takes this call (FP8, cols a
// multiple of 128, weights 16-byte aligned; the tensor-core GEMV's conditions)
bool signal_ok(const q35cu_weight *w, uint32_t cols, size_t in_bytes, size_t out_bytes)
{
    // read on every call, as launch_gemv reads Q35CU_GEMV_SIMT
    const bool simt = getenv("Q35CU_GEMV_SIMT") != nullptr;
    const char *e = getenv("Q35CU_HOST_SIGNAL");
    const bool off = e && atoi(e) == 0;
    return !simt && !off && w && w->kind == 0 && cols % 128 == 0 && (uintptr_t)w->d_w % 16 == 0 &&
           in_bytes <= ((size_t)64 << 20) && out_bytes <= kSignalOutMax;
}

}  // namespace

Q35_API void q35_mm_fp8(const uint8_t *W, const uint16_t *scale_bf16, uint32_t rows, uint32_t cols,
                        const float *x, float *y)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (rows == 0) return;
    const size_t nout = rows;
    if (!y) { set_error(Q35CU_ERR_ARG, "q35_mm_fp8: y is NULL"); float *o[1] = {nullptr}; fail_host(o, &nout, 1); return; }
    if (cols == 0) { memset(y, 0, (size_t)rows * 4); return; }
    int rc = Q35CU_OK;
    if (!W || !scale_bf16 || !x) rc = set_error(Q35CU_ERR_ARG, "q35_mm_fp8: NULL input");
    q35cu_weight *w = rc ? nullptr : cached_weight(0, W, scale_bf16, rows, cols);
    if (!rc && !w) rc = t_err;
    if (!rc && signal_ok(w, cols, (size_t)cols * 4, (size_t)rows * 4))
        rc = host_call_signal(
            x, (size_t)cols * 4, (size_t)rows * 4,
            [&](const float *dx, float *dy, cudaStream_t st, const HostSignal *sig) {
                GemvSeg g = seg_of(w, dy, rows);
                return launch_gemv(0, &g, 1, dx, cols, cols, 1, st, GemvTp{}, sig);
            },
            [&](const char *out) { memcpy(y, out, (size_t)rows * 4); });
    else if (!rc)
        rc = host_call(x, (size_t)cols * 4, y, (size_t)rows * 4, [&](const float *dx, float *dy, cudaStream_t st) {
            GemvSeg g = seg_of(w, dy, rows);
            return launch_gemv(0, &g, 1, dx, cols, cols, 1, st);
        });
    if (rc) { float *o[1] = {y}; fail_host(o, &nout, 1); }
}

Q35_API void q35_mm_fp8_batch(const uint8_t *W, const uint16_t *scale_bf16, uint32_t rows, uint32_t cols,
                              uint32_t n, const float *X, float *Y)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (rows == 0 || n == 0) return;
    const size_t nout = (size_t)rows * n;
    if (!Y) { set_error(Q35CU_ERR_ARG, "q35_mm_fp8_batch: Y is NULL"); float *o[1] = {nullptr}; fail_host(o, &nout, 1); return; }
    if (cols == 0) { memset(Y, 0, nout * 4); return; }
    int rc = Q35CU_OK;
    if (!W || !scale_bf16 || !X) rc = set_error(Q35CU_ERR_ARG, "q35_mm_fp8_batch: NULL input");
    q35cu_weight *w = rc ? nullptr : cached_weight(0, W, scale_bf16, rows, cols);
    if (!rc && !w) rc = t_err;
    // prefill-sized batches run the tensor-core GEMM on bf16-rounded
    // activations; multi-token decode batches run it on exact fp32
    // activations split hi/lo
    const bool tc = n >= gemm_min_tokens() && cols % 16 == 0;
    const bool tc_exact = !tc && n >= gemv_tc_min_tokens() && cols % 16 == 0;
    if (!rc && (tc || tc_exact)) {
        DevState *d = dev_state();
        const size_t xb = tc ? gemm_workspace_bytes(n, cols) : gemm_exact_workspace_bytes(n, cols);
        if (xb > d->xbf_cap) {
            if (d->d_xbf) dev_free(d->d_xbf, d->xbf_cap);
            d->d_xbf = nullptr;
            d->xbf_cap = 0;
            rc = dev_alloc(&d->d_xbf, xb);
            if (!rc) d->xbf_cap = xb;
        }
    }
    if (!rc && tc)
        rc = host_call(X, (size_t)n * cols * 4, Y, nout * 4, [&](const float *dx, float *dy, cudaStream_t st) {
            return launch_gemm_bf16(w, dx, true, n, dy, dev_state()->d_xbf, st);
        });
    else if (!rc && tc_exact)
        rc = host_call(X, (size_t)n * cols * 4, Y, nout * 4, [&](const float *dx, float *dy, cudaStream_t st) {
            return launch_gemm_exact(w, dx, n, dy, dev_state()->d_xbf, st);
        });
    else if (!rc && n <= 65535u * 4u && signal_ok(w, cols, (size_t)n * cols * 4, nout * 4))
        rc = host_call_signal(
            X, (size_t)n * cols * 4, nout * 4,
            [&](const float *dx, float *dy, cudaStream_t st, const HostSignal *sig) {
                GemvSeg g = seg_of(w, dy, rows);
                return launch_gemv(0, &g, 1, dx, cols, cols, n, st, GemvTp{}, sig);
            },
            [&](const char *out) { memcpy(Y, out, nout * 4); });
    else if (!rc)
        rc = host_call(X, (size_t)n * cols * 4, Y, nout * 4, [&](const float *dx, float *dy, cudaStream_t st) {
            GemvSeg g = seg_of(w, dy, rows);
            // token tiles of at most 64 per launch keep the grid's y extent small
            for (uint32_t t0 = 0; t0 < n; t0 += 65535u * 4u) {
                const uint32_t mt = n - t0 < 65535u * 4u ? n - t0 : 65535u * 4u;
                GemvSeg gt = g;
                gt.Y = dy + (size_t)t0 * rows;
                int r = launch_gemv(0, &gt, 1, dx + (size_t)t0 * cols, cols, cols, mt, st);
                if (r) return r;
            }
            return (int)Q35CU_OK;
        });
    if (rc) { float *o[1] = {Y}; fail_host(o, &nout, 1); }
}

Q35_API void q35_mm_fp8_multi4(const uint8_t *W[4], const uint16_t *sc[4], uint32_t rows[4], uint32_t cols,
                               const float *x, float *y[4])
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!W || !sc || !rows || !y) { set_error(Q35CU_ERR_ARG, "q35_mm_fp8_multi4: NULL array"); fail_host(nullptr, nullptr, 0); return; }
    uint32_t total = 0;
    for (int s = 0; s < 4; ++s) total += rows[s];
    if (total == 0) return;  // qwen35-c/src/q35_mm.c:187
    float *outs[4];
    size_t counts[4];
    for (int s = 0; s < 4; ++s) { outs[s] = rows[s] ? y[s] : nullptr; counts[s] = rows[s]; }
    if (cols == 0) { for (int s = 0; s < 4; ++s) if (rows[s]) memset(y[s], 0, (size_t)rows[s] * 4); return; }
    int rc = Q35CU_OK;
    q35cu_weight *ws[4] = {nullptr, nullptr, nullptr, nullptr};
    if (!x) rc = set_error(Q35CU_ERR_ARG, "q35_mm_fp8_multi4: x is NULL");
    for (int s = 0; s < 4 && !rc; ++s) {
        if (!rows[s]) continue;
        if (!W[s] || !sc[s] || !y[s]) { rc = set_error(Q35CU_ERR_ARG, "q35_mm_fp8_multi4: segment %d NULL", s); break; }
        ws[s] = cached_weight(0, W[s], sc[s], rows[s], cols);
        if (!ws[s]) rc = t_err;
    }
    if (!rc) {
        // outputs of the segments packed back to back in the staging area
        bool sig_ok = true;
        for (int s = 0; s < 4; ++s)
            if (ws[s] && !signal_ok(ws[s], cols, (size_t)cols * 4, (size_t)total * 4)) sig_ok = false;
        auto launch = [&](const float *dx, float *dy, cudaStream_t st, const HostSignal *sig) {
            GemvSeg segs[4];
            int n = 0;
            size_t off = 0;
            for (int s = 0; s < 4; ++s) {
                if (!ws[s]) continue;
                segs[n++] = seg_of(ws[s], dy + off, rows[s]);
                off += rows[s];
            }
            return launch_gemv(0, segs, n, dx, cols, cols, 1, st, GemvTp{}, sig);
        };
        auto scatter = [&](const char *out) {
            size_t off = 0;
            for (int s = 0; s < 4; ++s) {
                if (!ws[s]) continue;
                memcpy(y[s], reinterpret_cast<const float *>(out) + off, (size_t)rows[s] * 4);
                off += rows[s];
            }
        };
        if (sig_ok)
            rc = host_call_signal(x, (size_t)cols * 4, (size_t)total * 4, launch, scatter);
        else
            rc = host_call_ex(
                x, (size_t)cols * 4, (size_t)total * 4,
                [&](const float *dx, float *dy, cudaStream_t st) { return launch(dx, dy, st, nullptr); }, scatter);
    }
    if (rc) fail_host(outs, counts, 4);
}

Q35_API void q35_mm_bf16(const uint16_t *W, uint32_t rows, uint32_t cols, const float *x, float *y)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (rows == 0) return;
    const size_t nout = rows;
    if (!y) { set_error(Q35CU_ERR_ARG, "q35_mm_bf16: y is NULL"); float *o[1] = {nullptr}; fail_host(o, &nout, 1); return; }
    if (cols == 0) { memset(y, 0, (size_t)rows * 4); return; }
    int rc = Q35CU_OK;
    if (!W || !x) rc = set_error(Q35CU_ERR_ARG, "q35_mm_bf16: NULL input");
    q35cu_weight *w = rc ? nullptr : cached_weight(1, W, nullptr, rows, cols);
    if (!rc && !w) rc = t_err;
    if (!rc)
        rc = host_call(x, (size_t)cols * 4, y, (size_t)rows * 4, [&](const float *dx, float *dy, cudaStream_t st) {
            GemvSeg g = seg_of(w, dy, rows);
            return launch_gemv(1, &g, 1, dx, cols, cols, 1, st);
        });
    if (rc) { float *o[1] = {y}; fail_host(o, &nout, 1); }
}

// ------------------------------------------------------------------------
// tensor parallel: shard math (host only) and NCCL
// ------------------------------------------------------------------------
Q35_API int q35cu_shard_window(uint32_t rows, uint32_t cols, int mode, int rank, int world, uint32_t *row0,
                               uint32_t *nrows, uint32_t *col0, uint32_t *ncols)
{
    if (!row0 || !nrows || !col0 || !ncols) return set_error(Q35CU_ERR_ARG, "shard_window: NULL output");
    if (world < 1 || rank < 0 || rank >= world || !rows || !cols)
        return set_error(Q35CU_ERR_ARG, "shard_window: rank %d of %d, shape %ux%u", rank, world, rows, cols);
    const uint32_t dim = mode == Q35CU_SHARD_COLUMN ? rows : cols;
    const uint32_t blocks = (dim + 127) / 128;
    if ((uint32_t)world > blocks)
        return set_error(Q35CU_ERR_ARG, "shard_window: %u blocks cannot feed %d ranks", blocks, world);
    // equal 128-blocks per rank, the remainder spread over the first ranks
    const uint32_t per = blocks / world, extra = blocks % world;
    const uint32_t b0 = per * rank + (rank < (int)extra ? rank : extra);
    const uint32_t nb = per + (rank < (int)extra ? 1 : 0);
    uint32_t s0 = b0 * 128, len = nb * 128;
    if (s0 + len > dim) len = dim - s0;
    if (mode == Q35CU_SHARD_COLUMN) { *row0 = s0; *nrows = len; *col0 = 0; *ncols = cols; }
    else { *row0 = 0; *nrows = rows; *col0 = s0; *ncols = len; }
    return Q35CU_OK;
}

namespace {
ncclComm_t g_comm = nullptr;
int g_tp_rank = 0, g_tp_world = 1;

// NCCL is not a link-time dependency: a process that already holds a NCCL
// (torch's, for instance) keeps it, and one that never uses tensor
// parallelism never loads it.  Q35CU_NCCL_LIB names a library to dlopen
// when none is loaded yet.
struct Nccl {
    bool ok = false;
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRank) CommInitRank = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclAllReduce) AllReduce = nullptr;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
} g_nccl;

int load_nccl()
{
    if (g_nccl.ok) return Q35CU_OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) {
        const char *e = getenv("Q35CU_NCCL_LIB");
        h = dlopen(e && *e ? e : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) return set_error(Q35CU_ERR_NCCL, "cannot load NCCL: %s", dlerror());
#define Q35CU_SYM(n)                                                                   \
    g_nccl.n = reinterpret_cast<decltype(g_nccl.n)>(dlsym(h, "nccl" #n));              \
    if (!g_nccl.n) return set_error(Q35CU_ERR_NCCL, "NCCL lacks nccl%s", #n);
    Q35CU_SYM(GetUniqueId)
    Q35CU_SYM(CommInitRank)
    Q35CU_SYM(CommDestroy)
    Q35CU_SYM(AllReduce)
    Q35CU_SYM(AllGather)
    Q35CU_SYM(GetErrorString)
#undef Q35CU_SYM
    g_nccl.ok = true;
    return Q35CU_OK;
}

int nccl_err(ncclResult_t r, const char *what)
{
    return set_error(Q35CU_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "?");
}
}  // namespace

Q35_API int q35cu_nccl_unique_id(void *out, size_t cap)
{
    if (!out || cap < sizeof(ncclUniqueId)) return set_error(Q35CU_ERR_ARG, "nccl id needs %zu bytes", sizeof(ncclUniqueId));
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    ncclResult_t r = g_nccl.GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_err(r, "ncclGetUniqueId");
    memcpy(out, &id, sizeof id);
    return Q35CU_OK;
}

Q35_API int q35cu_tp_init(int rank, int world, const void *id, size_t idlen)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (!id || idlen < sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
        return set_error(Q35CU_ERR_ARG, "tp_init: rank %d world %d", rank, world);
    if (!dev_state()) return t_err;
    int rc = load_nccl();
    if (rc) return rc;
    if (g_comm) { g_nccl.CommDestroy(g_comm); g_comm = nullptr; }
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof uid);
    ncclResult_t r = g_nccl.CommInitRank(&g_comm, world, uid, rank);
    if (r != ncclSuccess) { g_comm = nullptr; return nccl_err(r, "ncclCommInitRank"); }
    g_tp_rank = rank;
    g_tp_world = world;
    return Q35CU_OK;
}

Q35_API int q35cu_tp_world(void) { return g_comm ? g_tp_world : 1; }
Q35_API int q35cu_tp_rank(void) { return g_comm ? g_tp_rank : 0; }

Q35_API int q35cu_tp_finalize(void)
{
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    if (g_comm) {
        ncclResult_t r = g_nccl.CommDestroy(g_comm);
        g_comm = nullptr;
        if (r != ncclSuccess) return nccl_err(r, "ncclCommDestroy");
    }
    g_tp_world = 1;
    g_tp_rank = 0;
    return Q35CU_OK;
}

Q35_API int q35cu_allreduce_f32(float *buf, size_t n, void *stream)
{
    if (!g_comm) return set_error(Q35CU_ERR_NCCL, "tensor parallel not initialised");
    ncclResult_t r = g_nccl.AllReduce(buf, buf, n, ncclFloat32, ncclSum, g_comm, pick(stream));
    return r == ncclSuccess ? Q35CU_OK : nccl_err(r, "ncclAllReduce");
}

Q35_API int q35cu_allgather_f32(const float *send, float *recv, size_t n_per_rank, void *stream)
{
    if (!g_comm) return set_error(Q35CU_ERR_NCCL, "tensor parallel not initialised");
    ncclResult_t r = g_nccl.AllGather(send, recv, n_per_rank, ncclFloat32, g_comm, pick(stream));
    return r == ncclSuccess ? Q35CU_OK : nccl_err(r, "ncclAllGather");
}
