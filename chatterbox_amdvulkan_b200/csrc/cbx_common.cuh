// cbx_common.cuh — shared device helpers and host launch plumbing of libcbx_ops.
//
// Everything here is sm_100a-only (the library is built with
// -gencode arch=compute_100a,code=sm_100a and nothing else).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cbx_ops.h"

namespace cbx {

// ------------------------------------------------------------ host side --

// Records `msg` (printf-style) as this thread's last error and returns `status`.
int fail(int status, const char* fmt, ...);
// Clears the thread's last error and returns CBX_OK.
int ok();
// Converts a CUDA error after a launch into CBX_ERR_LAUNCH with a message.
int launch_status(cudaError_t e, const char* what);

// Number of SMs of the current device (cached per device).
int num_sms();
// Programmatic dependent launch enabled (CBX_DISABLE_PDL unset or "0").
bool pdl_enabled();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool valid_type(int t) { return t == CBX_TYPE_F32 || t == CBX_TYPE_F16 || t == CBX_TYPE_BF16; }
__host__ __device__ inline int type_size(int t) { return t == CBX_TYPE_F32 ? 4 : 2; }

// Launches `kern` on `stream` with the programmatic-stream-serialization
// attribute (when enabled), so its launch overlaps the previous kernel's tail.
// Every kernel of the library calls grid_dep_wait() before it touches global
// memory (only L2 prefetches, which have no visible effect, come earlier),
// which keeps stream order for all data the kernel reads or writes; it
// signals grid_dep_launch() only after that wait, so at most one dependent
// kernel is resident ahead of the running one.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Resident CTAs per SM of kernel `fn` at `threads` threads / `smem` bytes on
// the current device (queried once per combination, then cached).
int occupancy_cached(const void* fn, int threads, size_t smem);

template <typename K>
int occupancy(K kern, int threads, size_t smem = 0) {
    return occupancy_cached(reinterpret_cast<const void*>(kern), threads, smem);
}

// Raises kernel `fn`'s dynamic shared memory limit to `smem` bytes on the
// current device (function attributes are per device; done once per device
// and kernel).  False when the driver refuses.
bool smem_opt_in_cached(const void* fn, size_t smem);

template <typename K>
bool smem_opt_in(K kern, size_t smem) {
    return smem_opt_in_cached(reinterpret_cast<const void*>(kern), smem);
}

// Device address of the library's device error word on the current device
// (bits CBX_DEVERR_*, read and cleared by cbx_device_errors).  Kernels in
// other translation units receive it as an argument.
int* device_error_word();

// ----------------------------------------------------------- device side --

// Programmatic dependent launch: wait until the preceding grid in the stream
// has completed and its memory is visible (no-op when launched without PDL).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid in the stream to start launching.
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a
// multiple of 16).  Kernels issue it for their inputs *before* grid_dep_wait:
// a prefetch has no visible effect (L2 is the point of coherence, so a line
// the preceding kernel writes afterwards is simply updated there), but when
// the inputs do not depend on that kernel their DRAM latency overlaps its
// tail instead of following it.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename T> struct Vec;  // elements per 16-byte vector
template <> struct Vec<float> { static constexpr int n = 4; };
template <> struct Vec<__nv_bfloat16> { static constexpr int n = 8; };
template <> struct Vec<__half> { static constexpr int n = 8; };

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// Unpack 32 bits holding 1 f32 or 2 16-bit elements.
__device__ __forceinline__ void unpack32(uint32_t w, float* f, float) { f[0] = __uint_as_float(w); }
__device__ __forceinline__ void unpack32(uint32_t w, float* f, __nv_bfloat16) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xffff0000u);
}
__device__ __forceinline__ void unpack32(uint32_t w, float* f, __half) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 t = __half22float2(h);
    f[0] = t.x;
    f[1] = t.y;
}
__device__ __forceinline__ uint32_t pack32(const float* f, float) { return __float_as_uint(f[0]); }
__device__ __forceinline__ uint32_t pack32(const float* f, __nv_bfloat16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[0], f[1]);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack32(const float* f, __half) {
    __half2 h = __floats2half2_rn(f[0], f[1]);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Loads N elements of T starting at p (N * sizeof(T) in {8, 16, 32} bytes; p
// aligned to min(16, N * sizeof(T))) and widens them to f32.
template <typename T, int N>
__device__ __forceinline__ void ldv(const T* p, float (&f)[N]) {
    constexpr int kBytes = N * (int)sizeof(T);
    constexpr int kPer32 = 4 / (int)sizeof(T);  // elements per 32-bit word
    static_assert(kBytes == 8 || kBytes == 16 || kBytes == 32, "vector size");
    if constexpr (kBytes == 8) {
        uint2 w = *reinterpret_cast<const uint2*>(p);
        unpack32(w.x, f + 0 * kPer32, T{});
        unpack32(w.y, f + 1 * kPer32, T{});
    } else {
#pragma unroll
        for (int q = 0; q < kBytes / 16; ++q) {
            uint4 w = *(reinterpret_cast<const uint4*>(p) + q);
            unpack32(w.x, f + (4 * q + 0) * kPer32, T{});
            unpack32(w.y, f + (4 * q + 1) * kPer32, T{});
            unpack32(w.z, f + (4 * q + 2) * kPer32, T{});
            unpack32(w.w, f + (4 * q + 3) * kPer32, T{});
        }
    }
}

// Rounds N f32 values to T (RNE) and stores them at p (alignment as ldv).
template <typename T, int N>
__device__ __forceinline__ void stv(T* p, const float (&f)[N]) {
    constexpr int kBytes = N * (int)sizeof(T);
    constexpr int kPer32 = 4 / (int)sizeof(T);
    static_assert(kBytes == 8 || kBytes == 16 || kBytes == 32, "vector size");
    if constexpr (kBytes == 8) {
        uint2 w;
        w.x = pack32(f + 0 * kPer32, T{});
        w.y = pack32(f + 1 * kPer32, T{});
        *reinterpret_cast<uint2*>(p) = w;
    } else {
#pragma unroll
        for (int q = 0; q < kBytes / 16; ++q) {
            uint4 w;
            w.x = pack32(f + (4 * q + 0) * kPer32, T{});
            w.y = pack32(f + (4 * q + 1) * kPer32, T{});
            w.z = pack32(f + (4 * q + 2) * kPer32, T{});
            w.w = pack32(f + (4 * q + 3) * kPer32, T{});
            *(reinterpret_cast<uint4*>(p) + q) = w;
        }
    }
}

// ------------------------------------------- mbarrier and bulk copies --
// ~2^24 polls of mbarrier.try_wait (each may suspend briefly): seconds, far
// beyond any bulk transfer, so only a broken transfer reaches it.
constexpr uint32_t kMaxPolls = 1u << 24;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Bounded wait for phase `parity` of `bar`; false when it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMaxPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Bulk async copy global -> this CTA's shared memory (cp.async.bulk, no
// tensor map, no multicast): both addresses 16-byte aligned, `bytes` a
// multiple of 16; completion is counted on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ------------------------------------------------ sin by Cody & Waite --
// x = k pi + r by Cody & Waite's additive reduction with pi split in three f32
// parts (P1 and P2 have 12 significant bits, so k P1 and k P2 are exact for
// |k| < 2^12; P1 + P2 + P3 - pi ~ 1e-17), then the odd Taylor polynomial of
// sin to r^15 on |r| <= pi/2 (truncation below 1e-11).  k is rounded with the
// 1.5 * 2^23 shift, so everything stays on the FMA pipe, and the shifted
// value's last mantissa bit is k's parity.  Valid for |x| < 12000 (|k| < 2^12);
// returns sin(r) = (-1)^k sin(x) and k mod 2 in *k_odd.
__device__ __forceinline__ float sin_cw_core(float x, uint32_t* k_odd) {
    constexpr float kInvPi = 0.318309886183790671538f;
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    const float kk = fmaf(x, kInvPi, kShift);
    *k_odd = __float_as_uint(kk) & 1u;
    const float k = __fsub_rn(kk, kShift);
    float r = fmaf(-k, 3.1416015625f, x);
    r = fmaf(-k, -8.907169103622437e-06f, r);
    r = fmaf(-k, -1.7411031505432106e-09f, r);
    const float r2 = r * r;
    float p = fmaf(r2, -1.0f / 1307674368000.0f, 1.0f / 6227020800.0f);  // r^15, r^13
    p = fmaf(r2, p, -1.0f / 39916800.0f);                                 // r^11
    p = fmaf(r2, p, 1.0f / 362880.0f);                                    // r^9
    p = fmaf(r2, p, -1.0f / 5040.0f);                                     // r^7
    p = fmaf(r2, p, 1.0f / 120.0f);                                       // r^5
    p = fmaf(r2, p, -1.0f / 6.0f);                                        // r^3
    return fmaf(r * r2, p, r);
}
// +-sin(x) (sign unspecified: for callers that square it); within 2 ulp of
// |sin(x)| rounded correctly on |x| < 12000, sinf beyond and for inf / NaN.
__device__ __forceinline__ float sin_up_to_sign(float x) {
    if (!(fabsf(x) < 12000.0f)) return sinf(x);
    uint32_t odd;
    return sin_cw_core(x, &odd);
}
// sin(x), same accuracy.
__device__ __forceinline__ float sin_cw(float x) {
    if (!(fabsf(x) < 12000.0f)) return sinf(x);
    uint32_t odd;
    const float s = sin_cw_core(x, &odd);
    return __uint_as_float(__float_as_uint(s) ^ (odd << 31));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------ activations --
// f32, written on the PTX approximation instructions (one MUFU op each):
//   ex2.approx.ftz.f32  2^a to a few ulp, subnormal results -> 0
//   rcp.approx.ftz.f32  1/a to ~1 ulp, rcp(inf) = 0
// with e^x = 2^(x log2 e).  Rounding x log2 e costs |x| 2^-24 relative in e^x,
// so over |x| <= 30 (where outputs are not tiny) every activation stays
// within ~2e-6 relative of the exact value, inside the parity bar of 1e-5
// relative / 1e-6 absolute; results that flush to 0 are below the absolute
// floor.  inf / NaN propagate as in the IEEE formula (x * 0 for x = -inf
// gives NaN, as the reference's x * tanh(...) / x * sigmoid(...) do).

__device__ __forceinline__ float ex2_approx(float a) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
}
__device__ __forceinline__ float rcp_approx(float a) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
}
constexpr float kLog2e = 1.4426950408889634f;

// GELU-tanh: 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3), through
// the identity 0.5 (1 + tanh(u)) = 1 / (1 + e^(-2u)): no cancellation in
// 1 + tanh(u) for negative x (where the f32 tanh form rounds tiny results to 0).
__device__ __forceinline__ float gelu_tanh_f(float x) {
    const float kC = 0.7978845608028654f;  // sqrt(2/pi)
    const float u = kC * fmaf(0.044715f * x, x * x, x);
    return x * rcp_approx(1.0f + ex2_approx(u * (-2.0f * kLog2e)));
}

// SiLU: x / (1 + e^-x).
__device__ __forceinline__ float silu_f(float x) {
    return x * rcp_approx(1.0f + ex2_approx(x * -kLog2e));
}

// Mish: x tanh(softplus(x)).  tanh(log(1 + e^x)) = n / (n + 2) with
// n = e^x (e^x + 2): one exponential and no cancellation for negative x.  The
// exponent is clamped at 20, where the reference's softplus becomes the
// identity and tanh rounds to 1: there n / (n + 2) = 1 - 9e-18, so y = x to
// within one f32 rounding (and n <= 2.4e17 cannot overflow).
__device__ __forceinline__ float mish_f(float x) {
    const float e = ex2_approx(fminf(x, 20.0f) * kLog2e);
    const float n = e * (e + 2.0f);
    return x * (n * rcp_approx(n + 2.0f));
}

// erfc(z) for z >= 0 by the Chebyshev fit of W. H. Press et al., Numerical
// Recipes (2nd ed., section 6.2, erfcc): erfc(z) = t exp(-z^2 + P(t)), t =
// 1 / (1 + z / 2), P of degree 9, fractional error below 1.2e-7 in exact
// arithmetic.  Evaluated in f32 (Horner by FMA, the exponential on ex2) it
// stays within 3.6e-6 relative for z <= 6 (checked on the CPU against double
// erfc); the error grows with the exponent's magnitude, i.e. where erfc is
// below 1e-15.  inf gives 0, NaN gives NaN.
__device__ __forceinline__ float erfc_nonneg(float z) {
    const float t = rcp_approx(fmaf(0.5f, z, 1.0f));
    float p = 0.17087277f;
    p = fmaf(t, p, -0.82215223f);
    p = fmaf(t, p, 1.48851587f);
    p = fmaf(t, p, -1.13520398f);
    p = fmaf(t, p, 0.27886807f);
    p = fmaf(t, p, -0.18628806f);
    p = fmaf(t, p, 0.09678418f);
    p = fmaf(t, p, 0.37409196f);
    p = fmaf(t, p, 1.00002368f);
    const float w = fmaf(-z, z, fmaf(t, p, -1.26551223f));
    return t * ex2_approx(w * kLog2e);
}

// Exact GELU 0.5 x (1 + erf(x / sqrt 2)) written as 0.5 x erfc(-x / sqrt 2):
// the same value without the cancellation of 1 + erf for negative x.  With
// a = |x| / sqrt 2: erfc(-x / sqrt 2) = erfc(a) for x <= 0 and 2 - erfc(a)
// for x > 0.
__device__ __forceinline__ float gelu_erf_f(float x) {
    const float e = erfc_nonneg(fabsf(x) * 0.70710678118654752f);
    return 0.5f * x * (x <= 0.0f ? e : 2.0f - e);
}

// ELU (alpha 1): x for x >= 0, e^x - 1 below (CUDA's full-precision expm1f).
__device__ __forceinline__ float elu_f(float x) { return x >= 0.0f ? x : expm1f(x); }

// Activations without a parameter (LeakyReLU's slope is applied by its caller).
template <int ACT>
__device__ __forceinline__ float act_f(float x) {
    if constexpr (ACT == CBX_ACT_MISH) return mish_f(x);
    else if constexpr (ACT == CBX_ACT_SILU) return silu_f(x);
    else if constexpr (ACT == CBX_ACT_GELU_TANH) return gelu_tanh_f(x);
    else if constexpr (ACT == CBX_ACT_GELU_ERF) return gelu_erf_f(x);
    else if constexpr (ACT == CBX_ACT_ELU) return elu_f(x);
    else return x;
}

// ---------------------------------------------- activations on f32 pairs --
// The same formulas as above for two values at once: the arithmetic on the
// packed f32x2 instructions (add / mul / fma .rn.f32x2, two IEEE f32
// operations each), the MUFU approximations and min per element.  Where the
// scalar form's add of a product may be contracted into an FMA, the pair form
// uses the packed FMA, so both round the same way.
__device__ __forceinline__ float2 pair(float v) { return make_float2(v, v); }

// The exponent -2 u log2(e), u = sqrt(2/pi) (x + 0.044715 x^3), is formed as
// x (K + 0.044715 K x^2) with K = -2 sqrt(2/pi) log2(e) folded at compile
// time: three packed operations per pair instead of five.  It rounds a few
// times fewer than the scalar form; the difference is a few ulp of the
// exponent, as in the scalar form's own error analysis above.
__device__ __forceinline__ float2 gelu_tanh_f2(float2 x) {
    constexpr float kK = (float)(-2.0 * 0.7978845608028654 * 1.4426950408889634);
    constexpr float kK3 = (float)(-2.0 * 0.7978845608028654 * 1.4426950408889634 * 0.044715);
    const float2 t = __fmul2_rn(x, __ffma2_rn(__fmul2_rn(x, x), pair(kK3), pair(kK)));
    const float2 d = __fadd2_rn(pair(1.0f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
    return __fmul2_rn(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}

__device__ __forceinline__ float2 silu_f2(float2 x) {
    const float2 t = __fmul2_rn(x, pair(-kLog2e));
    const float2 d = __fadd2_rn(pair(1.0f), make_float2(ex2_approx(t.x), ex2_approx(t.y)));
    return __fmul2_rn(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}

__device__ __forceinline__ float2 mish_f2(float2 x) {
    const float2 t = __fmul2_rn(make_float2(fminf(x.x, 20.0f), fminf(x.y, 20.0f)), pair(kLog2e));
    const float2 e = make_float2(ex2_approx(t.x), ex2_approx(t.y));
    const float2 n = __fmul2_rn(e, __fadd2_rn(e, pair(2.0f)));
    const float2 d = __fadd2_rn(n, pair(2.0f));
    return __fmul2_rn(x, __fmul2_rn(n, make_float2(rcp_approx(d.x), rcp_approx(d.y))));
}

// GELU-erf on a pair: erfc_nonneg's Horner steps and products on packed FMAs.
__device__ __forceinline__ float2 gelu_erf_f2(float2 x) {
    const float2 z = __fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), pair(0.70710678118654752f));
    const float2 q = __ffma2_rn(pair(0.5f), z, pair(1.0f));
    const float2 t = make_float2(rcp_approx(q.x), rcp_approx(q.y));
    float2 p = pair(0.17087277f);
    p = __ffma2_rn(t, p, pair(-0.82215223f));
    p = __ffma2_rn(t, p, pair(1.48851587f));
    p = __ffma2_rn(t, p, pair(-1.13520398f));
    p = __ffma2_rn(t, p, pair(0.27886807f));
    p = __ffma2_rn(t, p, pair(-0.18628806f));
    p = __ffma2_rn(t, p, pair(0.09678418f));
    p = __ffma2_rn(t, p, pair(0.37409196f));
    p = __ffma2_rn(t, p, pair(1.00002368f));
    const float2 w = __ffma2_rn(__fmul2_rn(z, pair(-1.0f)), z, __ffma2_rn(t, p, pair(-1.26551223f)));
    const float2 a = __fmul2_rn(w, pair(kLog2e));
    const float2 e = __fmul2_rn(t, make_float2(ex2_approx(a.x), ex2_approx(a.y)));
    const float2 c = make_float2(x.x <= 0.0f ? e.x : 2.0f - e.x, x.y <= 0.0f ? e.y : 2.0f - e.y);
    return __fmul2_rn(__fmul2_rn(pair(0.5f), x), c);
}

template <int ACT>
__device__ __forceinline__ float2 act_f2(float2 x) {
    if constexpr (ACT == CBX_ACT_GELU_ERF) return gelu_erf_f2(x);
    else if constexpr (ACT == CBX_ACT_MISH) return mish_f2(x);
    else if constexpr (ACT == CBX_ACT_SILU) return silu_f2(x);
    else if constexpr (ACT == CBX_ACT_GELU_TANH) return gelu_tanh_f2(x);
    else return make_float2(act_f<ACT>(x.x), act_f<ACT>(x.y));
}

}  // namespace cbx
