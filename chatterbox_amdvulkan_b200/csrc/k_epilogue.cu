// k_epilogue.cu — the elementwise neighbours of the engine's GEMMs and convs:
// bias add fused with an activation (T3 fc bias + GELU, CFM conv bias, HiFT
// ELU / LeakyReLU) and HiFT's three-ResBlock average.
//
// Both are one streaming pass (read x [+ bias], write y): HBM-bound at
// 2 x sizeof(T) bytes per element for cbx_bias_act, 4 x sizeof(T) for
// cbx_sum3_scale.  The bias add is rounded to f32 before the activation and
// the sum's three ggml nodes keep their separate f32 roundings
// (__fadd_rn / __fmul_rn), so cbx_sum3_scale is bit-exact with ggml's order.
#include "cbx_common.cuh"

namespace cbx {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;  // vectors per thread in the row kernel

template <int ACT>
__device__ __forceinline__ float act_p(float x, float p) {
    if constexpr (ACT == CBX_ACT_LEAKY_RELU) return x >= 0.0f ? x : x * p;
    else return act_f<ACT>(x);
}

// Rows of `hidden` elements with hidden % V == 0 and 16-byte alignment:
// blockIdx.x picks a chunk of kThreads * kUnroll vectors of a row, blockIdx.y
// the row (looping by gridDim.y), so no per-element index division is needed.
template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) k_bias_act_rows(const T* x, T* y, int64_t n_rows,
                                                            int hidden, const float* bias,
                                                            int axis, int64_t bias_len, float p) {
    constexpr int V = Vec<T>::n;
    const int vpr = hidden / V;
    const int vi0 = blockIdx.x * (kThreads * kUnroll) + threadIdx.x;
    if (threadIdx.x == 0 && blockIdx.y < n_rows && vi0 < vpr) {  // first chunk, before the wait
        const int nv = vpr - vi0 < kThreads * kUnroll ? vpr - vi0 : kThreads * kUnroll;
        prefetch_l2(x + (int64_t)blockIdx.y * hidden + (int64_t)vi0 * V, (uint32_t)nv * 16u);
    }
    grid_dep_wait();
    grid_dep_launch();
    for (int64_t r = blockIdx.y; r < n_rows; r += gridDim.y) {
        const T* xr = x + r * hidden;
        T* yr = y + r * hidden;
        const float rb = (bias && axis == CBX_BIAS_NE1) ? __ldg(bias + r % bias_len) : 0.0f;
        float f[kUnroll][V];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int vi = vi0 + u * kThreads;
            if (vi < vpr) ldv<T, V>(xr + (int64_t)vi * V, f[u]);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int vi = vi0 + u * kThreads;
            if (vi < vpr) {
                float b[V];
                if (bias && axis == CBX_BIAS_NE0) {
                    ldv<float, V>(bias + vi * V, b);
                } else {
#pragma unroll
                    for (int j = 0; j < V; ++j) b[j] = rb;
                }
                if constexpr (ACT == CBX_ACT_GELU_TANH || ACT == CBX_ACT_SILU ||
                              ACT == CBX_ACT_MISH) {
                    // the bias add (its own f32 rounding, as ggml_add) and the
                    // activation on packed f32 pairs
#pragma unroll
                    for (int j = 0; j < V; j += 2) {
                        const float2 r = act_f2<ACT>(__fadd2_rn(make_float2(f[u][j], f[u][j + 1]),
                                                                make_float2(b[j], b[j + 1])));
                        f[u][j] = r.x;
                        f[u][j + 1] = r.y;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < V; ++j) f[u][j] = act_p<ACT>(__fadd_rn(f[u][j], b[j]), p);
                }
                stv<T, V>(yr + (int64_t)vi * V, f[u]);
            }
        }
    }
}

// Any shape / alignment: flat grid-stride, column = e % hidden.
template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) k_bias_act_scalar(const T* x, T* y, int64_t n,
                                                              int64_t hidden, const float* bias,
                                                              int axis, int64_t bias_len, float p) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += stride) {
        float b = 0.0f;
        if (bias) b = axis == CBX_BIAS_NE0 ? bias[e % hidden] : bias[(e / hidden) % bias_len];
        y[e] = from_f<T>(act_p<ACT>(__fadd_rn(to_f(x[e]), b), p));
    }
}

// y = ((a + b) + c) * s, flat, 16-byte vectors (+ ragged tail).
template <typename T>
__global__ void __launch_bounds__(kThreads) k_sum3_vec(const T* a, const T* b, const T* c,
                                                       float s, T* y, int64_t n) {
    constexpr int V = Vec<T>::n;
    grid_dep_wait();
    grid_dep_launch();
    const int64_t nvec = n / V;
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec; i += stride) {
        float fa[V], fb[V], fc[V];
        ldv<T, V>(a + i * V, fa);
        ldv<T, V>(b + i * V, fb);
        ldv<T, V>(c + i * V, fc);
#pragma unroll
        for (int j = 0; j < V; ++j) fa[j] = __fmul_rn(__fadd_rn(__fadd_rn(fa[j], fb[j]), fc[j]), s);
        stv<T, V>(y + i * V, fa);
    }
    const int64_t tail = n - nvec * V;
    if (blockIdx.x == 0 && threadIdx.x < tail) {
        const int64_t e = nvec * V + threadIdx.x;
        y[e] = from_f<T>(__fmul_rn(__fadd_rn(__fadd_rn(to_f(a[e]), to_f(b[e])), to_f(c[e])), s));
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) k_sum3_scalar(const T* a, const T* b, const T* c,
                                                          float s, T* y, int64_t n) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += stride)
        y[e] = from_f<T>(__fmul_rn(__fadd_rn(__fadd_rn(to_f(a[e]), to_f(b[e])), to_f(c[e])), s));
}

template <typename T, int ACT>
int run_bias_act(const void* xv, void* yv, int64_t n_rows, int64_t hidden, const float* bias,
                 int axis, int64_t bias_len, float p, cudaStream_t st) {
    constexpr int V = Vec<T>::n;
    const T* x = static_cast<const T*>(xv);
    T* y = static_cast<T*>(yv);
    const bool vec = aligned16(x) && aligned16(y) && hidden % V == 0 && hidden <= INT32_MAX &&
                     (!bias || axis == CBX_BIAS_NE1 || aligned16(bias));
    cudaError_t e;
    if (vec) {
        const int64_t vpr = hidden / V;
        const int64_t chunks = (vpr + kThreads * kUnroll - 1) / (kThreads * kUnroll);
        const unsigned gy = (unsigned)(n_rows < 65535 ? n_rows : 65535);
        e = launch(k_bias_act_rows<T, ACT>, dim3((unsigned)chunks, gy), dim3(kThreads), 0, st, x, y,
                   n_rows, (int)hidden, bias, axis, bias_len, p);
    } else {
        const int64_t n = n_rows * hidden;
        int64_t blocks = (n + kThreads - 1) / kThreads;
        const int64_t cap = (int64_t)num_sms() * 8;
        if (blocks > cap) blocks = cap;
        e = launch(k_bias_act_scalar<T, ACT>, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, y,
                   n, hidden, bias, axis, bias_len, p);
    }
    return launch_status(e, "cbx_bias_act");
}

template <typename T>
int dispatch_act(const void* x, void* y, int64_t n_rows, int64_t hidden, const float* bias,
                 int axis, int64_t bias_len, int act, float p, cudaStream_t st) {
    switch (act) {
        case CBX_ACT_MISH: return run_bias_act<T, CBX_ACT_MISH>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
        case CBX_ACT_SILU: return run_bias_act<T, CBX_ACT_SILU>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
        case CBX_ACT_GELU_TANH: return run_bias_act<T, CBX_ACT_GELU_TANH>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
        case CBX_ACT_GELU_ERF: return run_bias_act<T, CBX_ACT_GELU_ERF>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
        case CBX_ACT_LEAKY_RELU: return run_bias_act<T, CBX_ACT_LEAKY_RELU>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
        case CBX_ACT_ELU: return run_bias_act<T, CBX_ACT_ELU>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
        default: return run_bias_act<T, CBX_ACT_NONE>(x, y, n_rows, hidden, bias, axis, bias_len, p, st);
    }
}

template <typename T>
int run_sum3(const void* av, const void* bv, const void* cv, float s, void* yv, int64_t n,
             cudaStream_t st) {
    const T* a = static_cast<const T*>(av);
    const T* b = static_cast<const T*>(bv);
    const T* c = static_cast<const T*>(cv);
    T* y = static_cast<T*>(yv);
    const int sms = num_sms();
    cudaError_t e;
    if (aligned16(a) && aligned16(b) && aligned16(c) && aligned16(y)) {
        int64_t blocks = (n / Vec<T>::n + kThreads - 1) / kThreads;
        if (blocks < 1) blocks = 1;
        const int64_t cap = (int64_t)sms * occupancy(k_sum3_vec<T>, kThreads);
        if (blocks > cap) blocks = cap;
        e = launch(k_sum3_vec<T>, dim3((unsigned)blocks), dim3(kThreads), 0, st, a, b, c, s, y, n);
    } else {
        int64_t blocks = (n + kThreads - 1) / kThreads;
        const int64_t cap = (int64_t)sms * 8;
        if (blocks > cap) blocks = cap;
        e = launch(k_sum3_scalar<T>, dim3((unsigned)blocks), dim3(kThreads), 0, st, a, b, c, s, y,
                   n);
    }
    return launch_status(e, "cbx_sum3_scale");
}

}  // namespace
}  // namespace cbx

extern "C" CBX_API int cbx_bias_act(const void* x, void* y, int type, int64_t n_rows,
                                    int64_t hidden, const float* bias, int bias_axis,
                                    int64_t bias_len, int act, float act_param,
                                    cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_bias_act";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n_rows < 0 || hidden <= 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_rows %lld hidden %lld", name, (long long)n_rows,
                    (long long)hidden);
    if (act < CBX_ACT_NONE || act > CBX_ACT_ELU)
        return fail(CBX_ERR_INVALID_ARG, "%s: act %d", name, act);
    if (bias_axis != CBX_BIAS_NE0 && bias_axis != CBX_BIAS_NE1)
        return fail(CBX_ERR_INVALID_ARG, "%s: bias_axis %d", name, bias_axis);
    if (bias && bias_axis == CBX_BIAS_NE0 && bias_len != hidden)
        return fail(CBX_ERR_INVALID_ARG, "%s: bias along ne0 needs bias_len == hidden", name);
    if (bias && bias_axis == CBX_BIAS_NE1 && bias_len <= 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: bias_len %lld", name, (long long)bias_len);
    if (!valid_type(type)) return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: type %d", name, type);
    if (n_rows == 0) return ok();
    if (!x || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL x or y", name);
    switch (type) {
        case CBX_TYPE_F32: return dispatch_act<float>(x, y, n_rows, hidden, bias, bias_axis, bias_len, act, act_param, st);
        case CBX_TYPE_BF16: return dispatch_act<__nv_bfloat16>(x, y, n_rows, hidden, bias, bias_axis, bias_len, act, act_param, st);
        default: return dispatch_act<__half>(x, y, n_rows, hidden, bias, bias_axis, bias_len, act, act_param, st);
    }
}

extern "C" CBX_API int cbx_sum3_scale(const void* a, const void* b, const void* c, float scale,
                                      void* y, int64_t n, int type, cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_sum3_scale";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n < 0) return fail(CBX_ERR_INVALID_ARG, "%s: n %lld", name, (long long)n);
    if (!valid_type(type)) return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: type %d", name, type);
    if (n == 0) return ok();
    if (!a || !b || !c || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL pointer", name);
    switch (type) {
        case CBX_TYPE_F32: return run_sum3<float>(a, b, c, scale, y, n, st);
        case CBX_TYPE_BF16: return run_sum3<__nv_bfloat16>(a, b, c, scale, y, n, st);
        default: return run_sum3<__half>(a, b, c, scale, y, n, st);
    }
}
