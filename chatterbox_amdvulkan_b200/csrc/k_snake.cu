// k_snake.cu — HiFT Snake, y = x + sin^2(alpha_c x) * alpha_inv_c, one pass.
//
// The engine runs this as five ggml nodes (hift_vocoder.cpp:64-73: mul, sin,
// sqr, mul, add) = five full passes; here it is one read and one write per
// element (8 bytes of HBM traffic).  The products keep ggml's node order and
// separate f32 roundings (__fmul_rn / __fadd_rn, no FMA contraction); the sin
// node's value is formed by sin_up_to_sign (|sin| suffices before sqr).
//
// [B][C][T] (PyTorch layout, alpha per row): 2-D grid, blockIdx.y walks rows
// (b, c), blockIdx.x a chunk of the row; alpha is uniform per CTA.
// [B][T][C] (engine layout, alpha along the contiguous axis): each thread owns
// a fixed group of four channels and walks rows (C <= 1024); wider rows use a
// flat grid where the channel of each 16-byte vector is its index mod C.
#include "cbx_common.cuh"

namespace cbx {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// |sin(x)| for the Snake's sin node, whose sign the following sqr node drops:
// Cody & Waite's reduction and a Taylor polynomial (sin_up_to_sign, within
// 2 ulp on |x| < 12000, sinf beyond).
__device__ __forceinline__ float snake_1(float x, float a, float ainv) {
    const float xa = __fmul_rn(x, a);
    const float s = sin_up_to_sign(xa);
    return __fadd_rn(x, __fmul_rn(__fmul_rn(s, s), ainv));
}

// snake_1 on two values at once: the same nodes, each an IEEE f32 operation
// on the packed f32x2 instructions (so the same roundings), and the same
// Cody & Waite reduction and polynomial; a lane whose argument is outside
// |x| < 12000 (or not finite) takes sinf as sin_up_to_sign does.
__device__ __forceinline__ float2 snake_2(float2 x, float2 a, float2 ainv) {
    constexpr float kInvPi = 0.318309886183790671538f;
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    const float2 xa = __fmul2_rn(x, a);
    const float2 kk = __ffma2_rn(xa, make_float2(kInvPi, kInvPi), make_float2(kShift, kShift));
    const float2 k = __fadd2_rn(kk, make_float2(-kShift, -kShift));
    const float2 nk = __fmul2_rn(k, make_float2(-1.0f, -1.0f));
    float2 r = __ffma2_rn(nk, make_float2(3.1416015625f, 3.1416015625f), xa);
    r = __ffma2_rn(nk, make_float2(-8.907169103622437e-06f, -8.907169103622437e-06f), r);
    r = __ffma2_rn(nk, make_float2(-1.7411031505432106e-09f, -1.7411031505432106e-09f), r);
    const float2 r2 = __fmul2_rn(r, r);
    float2 p = __ffma2_rn(r2, make_float2(-1.0f / 1307674368000.0f, -1.0f / 1307674368000.0f),
                          make_float2(1.0f / 6227020800.0f, 1.0f / 6227020800.0f));
    p = __ffma2_rn(r2, p, make_float2(-1.0f / 39916800.0f, -1.0f / 39916800.0f));
    p = __ffma2_rn(r2, p, make_float2(1.0f / 362880.0f, 1.0f / 362880.0f));
    p = __ffma2_rn(r2, p, make_float2(-1.0f / 5040.0f, -1.0f / 5040.0f));
    p = __ffma2_rn(r2, p, make_float2(1.0f / 120.0f, 1.0f / 120.0f));
    p = __ffma2_rn(r2, p, make_float2(-1.0f / 6.0f, -1.0f / 6.0f));
    float2 sn = __ffma2_rn(__fmul2_rn(r, r2), p, r);
    if (!(fabsf(xa.x) < 12000.0f)) sn.x = sinf(xa.x);
    if (!(fabsf(xa.y) < 12000.0f)) sn.y = sinf(xa.y);
    return __fadd2_rn(x, __fmul2_rn(__fmul2_rn(sn, sn), ainv));
}

__device__ __forceinline__ float4 snake_4(float4 v, float4 a, float4 ainv) {
    const float2 lo = snake_2(make_float2(v.x, v.y), make_float2(a.x, a.y), make_float2(ainv.x, ainv.y));
    const float2 hi = snake_2(make_float2(v.z, v.w), make_float2(a.z, a.w), make_float2(ainv.z, ainv.w));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float inv_alpha(const float* alpha_inv, const float* alpha, int c,
                                           float eps) {
    return alpha_inv ? __ldg(alpha_inv + c) : __fdiv_rn(1.0f, __fadd_rn(__ldg(alpha + c), eps));
}

// T % 4 == 0, 16-byte aligned.  Row r = blockIdx.y (+ k * gridDim.y).
__global__ void __launch_bounds__(kThreads) k_snake_bct_vec(const float* x, const float* alpha,
                                                            const float* alpha_inv, float eps,
                                                            int64_t rows, int C, int64_t T,
                                                            float* y) {
    const int64_t tv = T >> 2;  // float4 per row
    if (threadIdx.x == 0 && blockIdx.y < rows) {  // this CTA's first chunk, before the wait
        const int64_t v0 = (int64_t)blockIdx.x * (kThreads * kUnroll);
        if (v0 < tv) {
            const int64_t nv = tv - v0 < kThreads * kUnroll ? tv - v0 : kThreads * kUnroll;
            prefetch_l2(x + (int64_t)blockIdx.y * T + v0 * 4, (uint32_t)(nv * 16));
        }
    }
    grid_dep_wait();
    grid_dep_launch();  // next kernel may launch: this one is past its dependency
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const int c = (int)(r % C);
        const float a = __ldg(alpha + c);
        const float ainv = inv_alpha(alpha_inv, alpha, c, eps);
        const float4* xr = reinterpret_cast<const float4*>(x + r * T);
        float4* yr = reinterpret_cast<float4*>(y + r * T);
        const int64_t base = (int64_t)blockIdx.x * (kThreads * kUnroll) + threadIdx.x;
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = base + u * kThreads;
            if (i < tv) v[u] = xr[i];
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = base + u * kThreads;
            if (i < tv) {
                yr[i] = snake_4(v[u], make_float4(a, a, a, a), make_float4(ainv, ainv, ainv, ainv));
            }
        }
    }
}

// C % 4 == 0, 16-byte aligned: element index of vector i is 4i, channel 4i % C.
__global__ void __launch_bounds__(kThreads) k_snake_btc_vec(const float* x, const float* alpha,
                                                            const float* alpha_inv, float eps,
                                                            int64_t n, int C, float* y) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t nv = n >> 2;
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nv; i += stride) {
        const int c = (int)((i << 2) % C);
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        const float4 a = *reinterpret_cast<const float4*>(alpha + c);
        float4 ai;
        if (alpha_inv) {
            ai = *reinterpret_cast<const float4*>(alpha_inv + c);
        } else {
            ai.x = __fdiv_rn(1.0f, __fadd_rn(a.x, eps));
            ai.y = __fdiv_rn(1.0f, __fadd_rn(a.y, eps));
            ai.z = __fdiv_rn(1.0f, __fadd_rn(a.z, eps));
            ai.w = __fdiv_rn(1.0f, __fadd_rn(a.w, eps));
        }
        float4 o;
        o.x = snake_1(v.x, a.x, ai.x);
        o.y = snake_1(v.y, a.y, ai.y);
        o.z = snake_1(v.z, a.z, ai.z);
        o.w = snake_1(v.w, a.w, ai.w);
        reinterpret_cast<float4*>(y)[i] = o;
    }
}

// [B][T][C] with C % 4 == 0 and C / 4 <= kThreads: thread t owns the channel
// group vi = t % (C / 4) of row slot t / (C / 4), so alpha and alpha_inv for its
// four channels are loaded once.  CTA c takes the contiguous rows [c R, (c + 1) R),
// R = kUnroll row slots (at most 16 KB, prefetched into L2 before the PDL wait),
// all loaded before any math, no per-element division.
__global__ void __launch_bounds__(kThreads) k_snake_btc_rows(const float* x, const float* alpha,
                                                             const float* alpha_inv, float eps,
                                                             int64_t rows, int C,
                                                             int rows_per_cta, int64_t R,
                                                             float* y) {
    const int vpr = C >> 2;
    const int vi = threadIdx.x % vpr;
    const int slot = threadIdx.x / vpr;
    const int64_t r_lo = (int64_t)blockIdx.x * R;
    int64_t r_hi = r_lo + R;
    if (r_hi > rows) r_hi = rows;
    if (threadIdx.x == 0 && r_lo < r_hi) {
        const int64_t bytes = (r_hi - r_lo) * C * 4;
        prefetch_l2(x + r_lo * C, (uint32_t)(bytes < 16384 ? bytes : 16384));
    }
    grid_dep_wait();
    grid_dep_launch();
    if (slot >= rows_per_cta) return;
    const float4 a = *reinterpret_cast<const float4*>(alpha + 4 * vi);
    float4 ai;
    if (alpha_inv) {
        ai = *reinterpret_cast<const float4*>(alpha_inv + 4 * vi);
    } else {
        ai.x = __fdiv_rn(1.0f, __fadd_rn(a.x, eps));
        ai.y = __fdiv_rn(1.0f, __fadd_rn(a.y, eps));
        ai.z = __fdiv_rn(1.0f, __fadd_rn(a.z, eps));
        ai.w = __fdiv_rn(1.0f, __fadd_rn(a.w, eps));
    }
    const float4* xv = reinterpret_cast<const float4*>(x) + vi;
    float4* yv = reinterpret_cast<float4*>(y) + vi;
    for (int64_t r0 = r_lo + slot; r0 < r_hi; r0 += (int64_t)rows_per_cta * kUnroll) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t r = r0 + (int64_t)u * rows_per_cta;
            if (r < r_hi) v[u] = xv[r * vpr];
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t r = r0 + (int64_t)u * rows_per_cta;
            if (r < r_hi) {
                yv[r * vpr] = snake_4(v[u], a, ai);
            }
        }
    }
}

// Any shape / alignment, either layout.
__global__ void __launch_bounds__(kThreads) k_snake_scalar(const float* x, const float* alpha,
                                                           const float* alpha_inv, float eps,
                                                           int64_t n, int C, int64_t T, int bct,
                                                           float* y) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t stride = (int64_t)gridDim.x * kThreads;
    for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n; e += stride) {
        const int c = bct ? (int)((e / T) % C) : (int)(e % C);
        y[e] = snake_1(x[e], __ldg(alpha + c), inv_alpha(alpha_inv, alpha, c, eps));
    }
}

}  // namespace
}  // namespace cbx

extern "C" CBX_API int cbx_snake(const float* x, const float* alpha, const float* alpha_inv,
                                 float eps, int64_t B, int64_t C, int64_t T, int layout, float* y,
                                 cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_snake";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B < 0 || C <= 0 || T < 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: B %lld C %lld T %lld", name, (long long)B,
                    (long long)C, (long long)T);
    if (C > INT32_MAX) return fail(CBX_ERR_INVALID_ARG, "%s: C exceeds 2^31-1", name);
    if (layout != CBX_LAYOUT_BCT && layout != CBX_LAYOUT_BTC)
        return fail(CBX_ERR_INVALID_ARG, "%s: layout %d", name, layout);
    const int64_t n = B * C * T;
    if (n == 0) return ok();
    if (!x || !alpha || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL x, alpha or y", name);
    const int sms = num_sms();
    const bool al = aligned16(x) && aligned16(y);
    cudaError_t e;
    if (layout == CBX_LAYOUT_BCT && al && (T % 4) == 0) {
        const int64_t rows = B * C;
        const int64_t chunks = (T / 4 + kThreads * kUnroll - 1) / (kThreads * kUnroll);
        const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
        e = launch(k_snake_bct_vec, dim3((unsigned)chunks, gy), dim3(kThreads), 0, st, x, alpha,
                   alpha_inv, eps, rows, (int)C, T, y);
    } else if (layout == CBX_LAYOUT_BTC && al && (C % 4) == 0 && C / 4 <= kThreads &&
               aligned16(alpha) && (!alpha_inv || aligned16(alpha_inv))) {
        const int rpc = kThreads / (int)(C / 4);  // row slots per CTA
        const int64_t rows = B * T;
        // one pass per CTA: kUnroll rows per slot (<= 16 KB, all prefetched)
        const int64_t R = (int64_t)rpc * kUnroll;
        const int64_t blocks = (rows + R - 1) / R;
        if (blocks > INT32_MAX) return fail(CBX_ERR_INVALID_ARG, "%s: too many rows", name);
        e = launch(k_snake_btc_rows, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, alpha,
                   alpha_inv, eps, rows, (int)C, rpc, R, y);
    } else if (layout == CBX_LAYOUT_BTC && al && (C % 4) == 0 && aligned16(alpha) &&
               (!alpha_inv || aligned16(alpha_inv))) {
        int64_t blocks = (n / 4 + kThreads - 1) / kThreads;
        const int64_t cap = (int64_t)sms * 8;
        if (blocks > cap) blocks = cap;
        e = launch(k_snake_btc_vec, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, alpha,
                   alpha_inv, eps, n, (int)C, y);
    } else {
        int64_t blocks = (n + kThreads - 1) / kThreads;
        const int64_t cap = (int64_t)sms * 8;
        if (blocks > cap) blocks = cap;
        e = launch(k_snake_scalar, dim3((unsigned)blocks), dim3(kThreads), 0, st, x, alpha,
                   alpha_inv, eps, n, (int)C, T, layout == CBX_LAYOUT_BCT ? 1 : 0, y);
    }
    return launch_status(e, name);
}
