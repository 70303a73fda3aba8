// k_eltwise.cu — GELU-tanh, GELU-erf, SiLU and Mish over a flat buffer.
//
// One streaming pass: 16-byte vector loads, f32 math, one rounding at the
// store.  The grid is at most one wave of resident CTAs; each thread keeps
// kUnroll independent vectors in flight per iteration.  HBM-bound: 2 x
// sizeof(T) algorithmic bytes per element.
#include <stdlib.h>

#include "cbx_common.cuh"

namespace cbx {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// CBX_UNARY_CTAS_PER_SM caps the resident CTAs per SM of the vector kernel
// (leaves room for the next kernel's CTAs to launch early under PDL).
int ctas_per_sm_cap() {
    static const int v = [] {
        const char* e = getenv("CBX_UNARY_CTAS_PER_SM");
        return e ? atoi(e) : 0;
    }();
    return v;
}

template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) k_unary_vec(const T* x, T* y, int64_t n) {
    constexpr int V = Vec<T>::n;
    const int64_t nvec = n / V;
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    if (threadIdx.x < kUnroll) {  // this CTA's first chunks, before the wait
        const int64_t v0 = (int64_t)blockIdx.x * kThreads + threadIdx.x * stride;
        if (v0 < nvec) {
            const int64_t nv = nvec - v0 < kThreads ? nvec - v0 : kThreads;
            prefetch_l2(x + v0 * V, (uint32_t)(nv * 16));
        }
    }
    grid_dep_wait();
    grid_dep_launch();  // next kernel may launch: this one is past its dependency
    // Each iteration issues the loads of up to kUnroll vectors (those that
    // exist) before any compute, so a thread never waits on two round trips
    // in sequence when it owns more than one vector.
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec;
         i += kUnroll * stride) {
        float f[kUnroll][V];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            if (i + u * stride < nvec) ldv<T, V>(x + (i + u * stride) * V, f[u]);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            if (i + u * stride < nvec) {
#pragma unroll
                for (int k = 0; k < V; k += 2) {  // pairs: packed f32x2 arithmetic
                    const float2 r = act_f2<ACT>(make_float2(f[u][k], f[u][k + 1]));
                    f[u][k] = r.x;
                    f[u][k + 1] = r.y;
                }
                stv<T, V>(y + (i + u * stride) * V, f[u]);
            }
        }
    }
    // ragged tail (< V elements), handled by the first threads of block 0
    const int64_t tail = n - nvec * V;
    if (blockIdx.x == 0 && threadIdx.x < tail) {
        const int64_t e = nvec * V + threadIdx.x;
        y[e] = from_f<T>(act_f<ACT>(to_f(x[e])));
    }
}

// Any alignment: one element per thread-iteration.
template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) k_unary_scalar(const T* x, T* y, int64_t n) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += stride)
        y[e] = from_f<T>(act_f<ACT>(to_f(x[e])));
}

template <typename T, int ACT>
int run_unary(const void* xv, void* yv, int64_t n, cudaStream_t st, const char* name) {
    const T* x = static_cast<const T*>(xv);
    T* y = static_cast<T*>(yv);
    const int sms = num_sms();
    cudaError_t e;
    if (aligned16(x) && aligned16(y)) {
        auto kern = k_unary_vec<T, ACT>;
        const int occ = occupancy(kern, kThreads);  // cached per device
        const int64_t nvec = n / Vec<T>::n;
        int64_t blocks = (nvec + kThreads - 1) / kThreads;
        blocks = blocks < 1 ? 1 : blocks;
        // Small launches (under two full waves) keep at most 4 CTAs per SM, so
        // the next kernel's CTAs can become resident early and prefetch their
        // inputs under PDL; large ones use full occupancy.
        int per_sm = occ;
        if (blocks < 2LL * sms * occ && per_sm > 4) per_sm = 4;
        if (ctas_per_sm_cap() > 0 && ctas_per_sm_cap() < occ) per_sm = ctas_per_sm_cap();
        const int64_t cap = (int64_t)sms * per_sm;
        if (blocks > cap) blocks = cap;
        e = launch(kern, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, y, n);
    } else {
        auto kern = k_unary_scalar<T, ACT>;
        int64_t blocks = (n + kThreads - 1) / kThreads;
        const int64_t cap = (int64_t)sms * 8;
        if (blocks > cap) blocks = cap;
        e = launch(kern, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, y, n);
    }
    return launch_status(e, name);
}

template <int ACT>
int unary_entry(const void* x, void* y, int64_t n, int type, cbx_stream_t stream, const char* name) {
    if (n < 0) return fail(CBX_ERR_INVALID_ARG, "%s: n = %lld < 0", name, (long long)n);
    if (n == 0) return ok();
    if (!x || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL pointer", name);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (type) {
        case CBX_TYPE_F32: return run_unary<float, ACT>(x, y, n, st, name);
        case CBX_TYPE_BF16: return run_unary<__nv_bfloat16, ACT>(x, y, n, st, name);
        case CBX_TYPE_F16: return run_unary<__half, ACT>(x, y, n, st, name);
        default: return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: unsupported type %d", name, type);
    }
}

}  // namespace
}  // namespace cbx

extern "C" {

CBX_API int cbx_gelu_tanh(const void* x, void* y, int64_t n, int type, cbx_stream_t stream) {
    return cbx::unary_entry<CBX_ACT_GELU_TANH>(x, y, n, type, stream, "cbx_gelu_tanh");
}

CBX_API int cbx_silu(const void* x, void* y, int64_t n, int type, cbx_stream_t stream) {
    return cbx::unary_entry<CBX_ACT_SILU>(x, y, n, type, stream, "cbx_silu");
}

CBX_API int cbx_mish(const void* x, void* y, int64_t n, int type, cbx_stream_t stream) {
    return cbx::unary_entry<CBX_ACT_MISH>(x, y, n, type, stream, "cbx_mish");
}

CBX_API int cbx_gelu_erf(const void* x, void* y, int64_t n, int type, cbx_stream_t stream) {
    return cbx::unary_entry<CBX_ACT_GELU_ERF>(x, y, n, type, stream, "cbx_gelu_erf");
}

}  // extern "C"
