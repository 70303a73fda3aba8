// cbx_runtime.cu — error reporting, device queries, version and the host-side
// table builders of libcbx_ops.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "cbx_common.cuh"

#define CBX_VERSION_MAJOR 0
#define CBX_VERSION_MINOR 1
#define CBX_VERSION_PATCH 0

namespace cbx {

namespace {
thread_local char g_last_error[512] = {0};
constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices];
std::atomic<int> g_pdl{-1};
}  // namespace

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int ok() {
    g_last_error[0] = '\0';
    return CBX_OK;
}

int launch_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return ok();
    return fail(CBX_ERR_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
}

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) dev = 0;
    if (dev >= kMaxDevices) dev = kMaxDevices - 1;
    int n = g_sms[dev].load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;  // B200
        g_sms[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

int occupancy_cached(const void* fn, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, size_t, int>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    const auto key = std::make_tuple(fn, threads, smem, dev);
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess || n < 1)
        n = 1;
    std::lock_guard<std::mutex> g(mu);
    cache[key] = n;
    return n;
}

bool smem_opt_in_cached(const void* fn, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int>, size_t> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    const auto key = std::make_tuple(fn, dev);
    std::lock_guard<std::mutex> g(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= smem) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return false;
    done[key] = smem;
    return true;
}

bool pdl_enabled() {
    int v = g_pdl.load(std::memory_order_relaxed);
    if (v < 0) {
        const char* e = getenv("CBX_DISABLE_PDL");
        v = (e && e[0] && strcmp(e, "0") != 0) ? 0 : 1;
        g_pdl.store(v, std::memory_order_relaxed);
    }
    return v == 1;
}

}  // namespace cbx

extern "C" {

CBX_API int cbx_version(void) {
    return (CBX_VERSION_MAJOR << 16) | (CBX_VERSION_MINOR << 8) | CBX_VERSION_PATCH;
}

CBX_API const char* cbx_last_error(void) { return cbx::g_last_error; }

CBX_API const char* cbx_status_string(int status) {
    switch (status) {
        case CBX_OK: return "CBX_OK";
        case CBX_ERR_INVALID_ARG: return "CBX_ERR_INVALID_ARG";
        case CBX_ERR_UNSUPPORTED_DTYPE: return "CBX_ERR_UNSUPPORTED_DTYPE";
        case CBX_ERR_LAUNCH: return "CBX_ERR_LAUNCH";
        case CBX_ERR_INDEX_OOB: return "CBX_ERR_INDEX_OOB";
        case CBX_ERR_TIMEOUT: return "CBX_ERR_TIMEOUT";
        case CBX_ERR_CUDA: return "CBX_ERR_CUDA";
        default: return "CBX_ERR_UNKNOWN";
    }
}

// The engine's host loop (chatterbox-cpp/src/cfm_decoder.cpp:52-56), f32
// throughout: factor = logf(10000) / (half - 1); div_j = expf(-factor * j).
CBX_API int cbx_sinusoid_freqs(int32_t dim, float* freqs_host) {
    if (!freqs_host) return cbx::fail(CBX_ERR_INVALID_ARG, "cbx_sinusoid_freqs: freqs_host is NULL");
    if (dim < 4)
        return cbx::fail(CBX_ERR_INVALID_ARG, "cbx_sinusoid_freqs: dim %d < 4 (half - 1 must be > 0)",
                         (int)dim);
    const int half = dim / 2;
    const float log10000 = logf(10000.0f);
    const float factor = log10000 / (float)(half - 1);
    for (int j = 0; j < half; ++j) freqs_host[j] = expf(-factor * (float)j);
    return cbx::ok();
}

// chatterbox-cpp/src/hift_vocoder.cpp:419-420: v[i] = 1.0f / (a[i] + snake_eps).
CBX_API int cbx_snake_alpha_inv(const float* alpha_host, int64_t n, float eps,
                                float* alpha_inv_host) {
    if (!alpha_host || !alpha_inv_host || n < 0)
        return cbx::fail(CBX_ERR_INVALID_ARG, "cbx_snake_alpha_inv: bad arguments");
    for (int64_t i = 0; i < n; ++i) alpha_inv_host[i] = 1.0f / (alpha_host[i] + eps);
    return cbx::ok();
}

}  // extern "C"
