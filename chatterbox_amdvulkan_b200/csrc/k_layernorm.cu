// k_layernorm.cu — residual add fused with LayerNorm over ne0 (row-wise),
// with an optional fused activation and per-row mask (the engine-native
// [T][C] CausalBlock1D tail of the CFM estimator).
//
// One warp per row.  The row (x + resid) is read once with 16-byte vector
// loads into registers; mean and biased variance are computed two-pass from
// the registers (f32, warp-shuffle reductions), then s and y are written.
// HBM-bound: per row (2 + [resid]) reads and (1 + [sum_out]) writes of
// hidden elements, plus gamma/beta (L1/L2-resident across rows).
#include <stdlib.h>

#include <type_traits>

#include "cbx_common.cuh"

namespace cbx {
namespace {

// CBX_LN_WARP_ROWS=1 keeps the warp-per-row kernel for small row counts too
// (A/B measurements).
bool force_warp_rows() {
    static const bool v = [] {
        const char* e = getenv("CBX_LN_WARP_ROWS");
        return e && e[0] && e[0] != '0';
    }();
    return v;
}

int cta_nv_override() {
    static const int v = [] {
        const char* e = getenv("CBX_LN_CTA_NV");
        return e ? atoi(e) : 0;
    }();
    return v;
}

struct LnArgs {
    const void* x;
    const void* r;
    int64_t in_stride;
    const float* g;
    const float* b;
    float eps;
    int64_t n_rows;
    int H;
    void* s;
    void* y;
    int64_t out_stride;
    const float* mask;
};

// Vectorised path: hidden % V == 0, 16-byte aligned rows, hidden <= MAXV*32*V.
// PRE (used when there are too few rows to fill the GPU, so each warp's
// latency chain is the kernel's duration): gamma / beta are fetched right
// after the row's loads are issued, so their L2 round trip overlaps the DRAM
// latency of x / resid instead of following the statistics.  Without PRE the
// kernel needs half the registers and relies on occupancy to hide latency.
// gamma / beta are read through __restrict__ pointers (outputs never alias them).
template <typename Tin, typename Tout, int MAXV, int ACT, bool PRE, int MINB = 1>
__global__ void __launch_bounds__(256, MINB) k_ln_rows_vec(LnArgs a) {
    constexpr int V = Vec<Tin>::n;
    constexpr bool kPrefetchAffine = PRE && MAXV * V <= 32;  // <= 64 registers of gamma/beta
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int nvec = a.H / V;
    const float inv_h = 1.0f / (float)a.H;
    const Tin* X = static_cast<const Tin*>(a.x);
    const Tin* R = static_cast<const Tin*>(a.r);
    Tin* S = static_cast<Tin*>(a.s);
    Tout* Y = static_cast<Tout*>(a.y);
    const float* __restrict__ G = a.g;
    const float* __restrict__ Bt = a.b;
    const uint32_t row_bytes = (uint32_t)a.H * sizeof(Tin);
    const int64_t first = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    // L2 prefetch of this warp's first row (and of gamma / beta by the CTA's
    // first warp) before waiting on the preceding kernel.
    if (first < a.n_rows) {
        if (lane == 0) prefetch_l2(X + first * a.in_stride, row_bytes);
        if (lane == 1 && R) prefetch_l2(R + first * a.in_stride, row_bytes);
    }
    if (threadIdx.x == 2 && G) prefetch_l2(G, (uint32_t)a.H * 4);
    if (threadIdx.x == 3 && Bt) prefetch_l2(Bt, (uint32_t)a.H * 4);
    grid_dep_wait();
    grid_dep_launch();  // next kernel may launch: this one is past its dependency

    for (int64_t row = first; row < a.n_rows; row += nwarps) {
        float v[MAXV][V];
        float w[PRE ? MAXV : 1][V];
        const Tin* xr = X + row * a.in_stride;
        const Tin* rr = R ? R + row * a.in_stride : nullptr;
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            const int vi = k * 32 + lane;
            if (vi < nvec) {
                ldv<Tin, V>(xr + (int64_t)vi * V, v[k]);
                if constexpr (PRE) {
                    if (rr) ldv<Tin, V>(rr + (int64_t)vi * V, w[k]);
                }
            }
        }
        if constexpr (!PRE) {
            // load-and-add: the residual needs no second register array
            if (rr) {
#pragma unroll
                for (int k = 0; k < MAXV; ++k) {
                    const int vi = k * 32 + lane;
                    if (vi < nvec) {
                        float t[V];
                        ldv<Tin, V>(rr + (int64_t)vi * V, t);
#pragma unroll
                        for (int j = 0; j < V; ++j) v[k][j] += t[j];
                    }
                }
            }
        }
        float gg[kPrefetchAffine ? MAXV : 1][V], bb[kPrefetchAffine ? MAXV : 1][V];
        if constexpr (kPrefetchAffine) {
#pragma unroll
            for (int k = 0; k < MAXV; ++k) {
                const int vi = k * 32 + lane;
                if (vi < nvec) {
                    if (G) ldv<float, V>(G + vi * V, gg[k]);
                    if (Bt) ldv<float, V>(Bt + vi * V, bb[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            const int vi = k * 32 + lane;
#pragma unroll
            for (int j = 0; j < V; ++j) {
                if (vi >= nvec) v[k][j] = 0.0f;
                else if constexpr (PRE) {
                    if (rr) v[k][j] += w[k][j];
                }
            }
        }
        // mean: per-vector partial sums, then across vectors, then the warp
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            float p = 0.0f;
#pragma unroll
            for (int j = 0; j < V; ++j) p += v[k][j];
            sum += p;
        }
        const float mean = warp_sum(sum) * inv_h;
        float sq = 0.0f;
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            if (k * 32 + lane < nvec) {
                float p = 0.0f;
#pragma unroll
                for (int j = 0; j < V; ++j) {
                    const float d = v[k][j] - mean;
                    p = fmaf(d, d, p);
                }
                sq += p;
            }
        }
        const float var = warp_sum(sq) * inv_h;
        const float rstd = 1.0f / sqrtf(var + a.eps);
        const float m = a.mask ? a.mask[row] : 1.0f;

        Tin* sr = S ? S + row * a.out_stride : nullptr;
        Tout* yr = Y + row * a.out_stride;
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            const int vi = k * 32 + lane;
            if (vi < nvec) {
                float g2[V], b2[V], o[V];
                if constexpr (kPrefetchAffine) {
#pragma unroll
                    for (int j = 0; j < V; ++j) {
                        g2[j] = G ? gg[k][j] : 1.0f;
                        b2[j] = Bt ? bb[k][j] : 0.0f;
                    }
                } else {
                    if (G) ldv<float, V>(G + vi * V, g2);
                    else {
#pragma unroll
                        for (int j = 0; j < V; ++j) g2[j] = 1.0f;
                    }
                    if (Bt) ldv<float, V>(Bt + vi * V, b2);
                    else {
#pragma unroll
                        for (int j = 0; j < V; ++j) b2[j] = 0.0f;
                    }
                }
#pragma unroll
                for (int j = 0; j < V; ++j) {
                    float t = fmaf((v[k][j] - mean) * rstd, g2[j], b2[j]);
                    if constexpr (ACT != CBX_ACT_NONE) t = act_f<ACT>(t);
                    o[j] = t * m;
                }
                if (sr) stv<Tin, V>(sr + (int64_t)vi * V, v[k]);
                stv<Tout, V>(yr + (int64_t)vi * V, o);
            }
        }
    }
}

// Latency-bound regime (too few rows to fill the GPU): one CTA per row
// (grid = n_rows), NV 16-byte vectors per thread (blockDim = hidden / (V NV),
// a multiple of 32), so each thread's dependent instruction chain is short.
// Statistics in one reduction: each thread forms (mean, M2) of its NV*V
// values two-pass in registers; the pairs are merged with Chan's equal-count
// update (mean = (m_a + m_b) / 2, M2 = M2_a + M2_b + n/2 (m_b - m_a)^2) up a
// shuffle tree and then across the warps through shared memory: one barrier.
// gamma / beta and the row are prefetched to L2 before waiting on the
// preceding kernel and loaded together with the row.  RES / AFF select the
// residual input and the affine at compile time.
template <typename Tin, typename Tout, int NV, int ACT, bool RES, bool AFF>
__global__ void __launch_bounds__(512) k_ln_row_cta(LnArgs a) {
    constexpr int V = Vec<Tin>::n;
    constexpr int kPer = NV * V;  // values per thread
    __shared__ float2 red[16];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t row = blockIdx.x;
    const Tin* xr = static_cast<const Tin*>(a.x) + row * a.in_stride;
    const Tin* rr = RES ? static_cast<const Tin*>(a.r) + row * a.in_stride : nullptr;
    const float* __restrict__ G = a.g;
    const float* __restrict__ Bt = a.b;
    const uint32_t row_bytes = (uint32_t)a.H * sizeof(Tin);
    if (tid == 0) prefetch_l2(xr, row_bytes);
    if (RES && tid == 1) prefetch_l2(rr, row_bytes);
    if (AFF && tid == 2) prefetch_l2(G, (uint32_t)a.H * 4);
    if (AFF && tid == 3) prefetch_l2(Bt, (uint32_t)a.H * 4);
    grid_dep_wait();
    grid_dep_launch();  // next kernel may launch: this one is past its dependency

    float v[NV][V], w[NV][V], gg[NV][V], bb[NV][V];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int e = (k * blockDim.x + tid) * V;
        ldv<Tin, V>(xr + e, v[k]);
        if constexpr (RES) ldv<Tin, V>(rr + e, w[k]);
        if constexpr (AFF) {
            ldv<float, V>(G + e, gg[k]);
            ldv<float, V>(Bt + e, bb[k]);
        }
    }
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            if constexpr (RES) v[k][j] += w[k][j];
            m += v[k][j];
        }
    }
    // the residual sum needs no statistics: its stores drain while the row
    // is reduced (measured 0.1 us of the 2.3 us launch period at 256 x 1024)
    Tin* sr = a.s ? static_cast<Tin*>(a.s) + row * a.out_stride : nullptr;
    if (sr) {
#pragma unroll
        for (int k = 0; k < NV; ++k) stv<Tin, V>(sr + (k * blockDim.x + tid) * V, v[k]);
    }
    m *= 1.0f / (float)kPer;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const float d = v[k][j] - m;
            q = fmaf(d, d, q);
        }
    }
    float half_n = 0.5f * (float)kPer;  // n / 2 for two halves of n values each
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, o);
        const float qo = __shfl_xor_sync(0xffffffffu, q, o);
        const float d = mo - m;
        q = q + qo + half_n * d * d;
        m = 0.5f * (m + mo);
        half_n *= 2.0f;
    }
    const int nw = blockDim.x >> 5;
    const float inv_nw = 1.0f / (float)nw, inv_h = 1.0f / (float)a.H;  // off the critical path
    if (lane == 0) red[warp] = make_float2(m, q);
    __syncthreads();
    float mean = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (i < nw) mean += red[i].x;
    mean *= inv_nw;
    float m2 = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        if (i < nw) {
            const float2 t = red[i];
            const float d = t.x - mean;
            m2 += t.y + (32.0f * kPer) * d * d;
        }
    }
    const float rstd = rsqrtf(m2 * inv_h + a.eps);
    const float mk = a.mask ? a.mask[row] : 1.0f;
    Tout* yr = static_cast<Tout*>(a.y) + row * a.out_stride;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int e = (k * blockDim.x + tid) * V;
        float o[V];
#pragma unroll
        for (int j = 0; j < V; ++j) {
            float t = (v[k][j] - mean) * rstd;
            if constexpr (AFF) t = fmaf(t, gg[k][j], bb[k][j]);
            if constexpr (ACT != CBX_ACT_NONE) t = act_f<ACT>(t);
            o[j] = t * mk;
        }
        stv<Tout, V>(yr + e, o);
    }
}

// Any hidden size / alignment: one warp per row, three passes over the row
// (sum, squared deviations, write), the re-reads served by L1.
template <typename Tin, typename Tout, int ACT>
__global__ void __launch_bounds__(256) k_ln_rows_generic(LnArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const Tin* X = static_cast<const Tin*>(a.x);
    const Tin* R = static_cast<const Tin*>(a.r);
    Tin* S = static_cast<Tin*>(a.s);
    Tout* Y = static_cast<Tout*>(a.y);
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < a.n_rows;
         row += nwarps) {
        const Tin* xr = X + row * a.in_stride;
        const Tin* rr = R ? R + row * a.in_stride : nullptr;
        float sum = 0.0f;
        for (int j = lane; j < a.H; j += 32) sum += to_f(xr[j]) + (rr ? to_f(rr[j]) : 0.0f);
        const float mean = warp_sum(sum) / (float)a.H;
        float sq = 0.0f;
        for (int j = lane; j < a.H; j += 32) {
            const float d = (to_f(xr[j]) + (rr ? to_f(rr[j]) : 0.0f)) - mean;
            sq = fmaf(d, d, sq);
        }
        const float rstd = 1.0f / sqrtf(warp_sum(sq) / (float)a.H + a.eps);
        const float m = a.mask ? a.mask[row] : 1.0f;
        Tin* sr = S ? S + row * a.out_stride : nullptr;
        Tout* yr = Y + row * a.out_stride;
        for (int j = lane; j < a.H; j += 32) {
            const float sv = to_f(xr[j]) + (rr ? to_f(rr[j]) : 0.0f);
            float t = (sv - mean) * rstd;
            t = fmaf(t, a.g ? a.g[j] : 1.0f, a.b ? a.b[j] : 0.0f);
            if constexpr (ACT != CBX_ACT_NONE) t = act_f<ACT>(t);
            if (sr) sr[j] = from_f<Tin>(sv);
            yr[j] = from_f<Tout>(t * m);
        }
    }
}

template <typename K>
int launch_rows(K kern, const LnArgs& a, cudaStream_t st, const char* name) {
    const int sms = num_sms();
    int wpc;  // warps per CTA: spread small row counts over all SMs
    if (a.n_rows >= (int64_t)sms * 16) wpc = 8;
    else if (a.n_rows >= (int64_t)sms * 4) wpc = 4;
    else if (a.n_rows >= (int64_t)sms * 2) wpc = 2;
    else wpc = 1;
    const int threads = wpc * 32;
    const int occ = occupancy(kern, threads);
    int64_t blocks = (a.n_rows + wpc - 1) / wpc;
    const int64_t cap = (int64_t)sms * occ;
    if (blocks > cap) blocks = cap;
    if (blocks == cap) {
        // more rows than resident warps: the fewest CTAs that give every warp
        // the same number of rows (within one), so no last round of rows runs
        // on a fraction of the warps
        const int64_t rpw = (a.n_rows + cap * wpc - 1) / (cap * wpc);
        blocks = (a.n_rows + rpw * wpc - 1) / (rpw * wpc);
    }
    if (blocks < 1) blocks = 1;
    return launch_status(launch(kern, dim3((unsigned)blocks), dim3(threads), 0, st, a), name);
}

template <typename Tin, typename Tout, int ACT, bool PRE>
int dispatch_vec(const LnArgs& a, int per_lane, cudaStream_t st, const char* name) {
    if (per_lane <= 2) return launch_rows(k_ln_rows_vec<Tin, Tout, 2, ACT, PRE>, a, st, name);
    // MAXV 4 without the affine prefetch: bounded to 64 registers, 4 CTAs per SM
    // (80 unbounded, 3 per SM; bf16 configs[2] 97.3 -> 96.7 us, 8192 rows 12.3 -> 11.6 us).
    // 16-bit in with f32 out keeps its registers (it would spill under the bound).
    constexpr bool kWide = sizeof(Tin) < sizeof(Tout);
    if (per_lane <= 4)
        return launch_rows(k_ln_rows_vec<Tin, Tout, 4, ACT, PRE, (PRE || kWide) ? 1 : 4>, a, st, name);
    if (per_lane <= 8) return launch_rows(k_ln_rows_vec<Tin, Tout, 8, ACT, PRE>, a, st, name);
    return launch_rows(k_ln_rows_vec<Tin, Tout, 16, ACT, PRE>, a, st, name);
}

template <typename Tin, typename Tout, int ACT>
int dispatch_rows(const LnArgs& a, bool vec_ok, cudaStream_t st, const char* name) {
    constexpr int V = Vec<Tin>::n;
    const int sms = num_sms();
    if (vec_ok && a.n_rows <= (int64_t)sms * 4 && !force_warp_rows()) {
        // one CTA per row with nv vectors per thread (32..512 threads): 2 by
        // default; CBX_LN_CTA_NV=1|2|4 overrides it where the shape allows.
        const int nvec = a.H / V;
        int nv = 0;
        const int want = cta_nv_override();
        if (want == 4 && nvec % 128 == 0 && nvec / 4 <= 512) nv = 4;
        else if (want == 1 && nvec % 32 == 0 && nvec <= 512) nv = 1;
        else if (nvec % 64 == 0 && nvec / 2 <= 512) nv = 2;
        else if (nvec % 32 == 0 && nvec <= 512) nv = 1;
        // the affine template needs both gamma and beta (or neither)
        if (nv && (a.g == nullptr) == (a.b == nullptr)) {
            const dim3 grid((unsigned)a.n_rows), block((unsigned)(nvec / nv));
            cudaError_t e;
            const bool res = a.r != nullptr, aff = a.g != nullptr;
#define CBX_LN_CTA(NV_, R_, A_) launch(k_ln_row_cta<Tin, Tout, NV_, ACT, R_, A_>, grid, block, 0, st, a)
            if (nv == 4) {
                e = res ? (aff ? CBX_LN_CTA(4, true, true) : CBX_LN_CTA(4, true, false))
                        : (aff ? CBX_LN_CTA(4, false, true) : CBX_LN_CTA(4, false, false));
            } else if (nv == 2) {
                e = res ? (aff ? CBX_LN_CTA(2, true, true) : CBX_LN_CTA(2, true, false))
                        : (aff ? CBX_LN_CTA(2, false, true) : CBX_LN_CTA(2, false, false));
            } else {
                e = res ? (aff ? CBX_LN_CTA(1, true, true) : CBX_LN_CTA(1, true, false))
                        : (aff ? CBX_LN_CTA(1, false, true) : CBX_LN_CTA(1, false, false));
            }
#undef CBX_LN_CTA
            return launch_status(e, name);
        }
    }
    if (vec_ok) {
        const int per_lane = (a.H / V + 31) / 32;
        // fewer rows than ~16 warps per SM: latency-bound, prefetch the affine
        if (a.n_rows < (int64_t)num_sms() * 16)
            return dispatch_vec<Tin, Tout, ACT, true>(a, per_lane, st, name);
        return dispatch_vec<Tin, Tout, ACT, false>(a, per_lane, st, name);
    }
    return launch_rows(k_ln_rows_generic<Tin, Tout, ACT>, a, st, name);
}

template <typename Tin, typename Tout>
int dispatch_act(const LnArgs& a, int act, bool vec_ok, cudaStream_t st, const char* name) {
    if constexpr (std::is_same<Tin, float>::value && std::is_same<Tout, float>::value) {
        switch (act) {
            case CBX_ACT_MISH: return dispatch_rows<float, float, CBX_ACT_MISH>(a, vec_ok, st, name);
            case CBX_ACT_SILU: return dispatch_rows<float, float, CBX_ACT_SILU>(a, vec_ok, st, name);
            case CBX_ACT_GELU_TANH:
                return dispatch_rows<float, float, CBX_ACT_GELU_TANH>(a, vec_ok, st, name);
            default: return dispatch_rows<float, float, CBX_ACT_NONE>(a, vec_ok, st, name);
        }
    } else {
        if (act != CBX_ACT_NONE)
            return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: fused activation needs f32 in/out", name);
        return dispatch_rows<Tin, Tout, CBX_ACT_NONE>(a, vec_ok, st, name);
    }
}

template <typename Tin>
int dispatch_out(const LnArgs& a, int out_type, int act, bool vec_ok, cudaStream_t st,
                 const char* name) {
    switch (out_type) {
        case CBX_TYPE_F32: return dispatch_act<Tin, float>(a, act, vec_ok, st, name);
        case CBX_TYPE_BF16: return dispatch_act<Tin, __nv_bfloat16>(a, act, vec_ok, st, name);
        case CBX_TYPE_F16: return dispatch_act<Tin, __half>(a, act, vec_ok, st, name);
        default: return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: out_type %d", name, out_type);
    }
}

}  // namespace

// Shared by cbx_add_layernorm and the BTC form of cbx_layernorm_channels.
int row_layernorm(const void* x, const void* r, int in_type, int64_t in_stride, const float* g,
                  const float* b, float eps, int64_t n_rows, int64_t H, void* s, void* y,
                  int out_type, int64_t out_stride, int act, const float* mask, cudaStream_t st,
                  const char* name) {
    if (n_rows < 0 || H <= 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_rows %lld / hidden %lld", name, (long long)n_rows,
                    (long long)H);
    if (H > (int64_t)1 << 30) return fail(CBX_ERR_INVALID_ARG, "%s: hidden too large", name);
    if (!(eps >= 0.0f)) return fail(CBX_ERR_INVALID_ARG, "%s: eps must be >= 0", name);
    if (in_stride == 0) in_stride = H;
    if (out_stride == 0) out_stride = H;
    if (in_stride < H || out_stride < H)
        return fail(CBX_ERR_INVALID_ARG, "%s: row stride smaller than hidden", name);
    if (!valid_type(in_type) || !valid_type(out_type))
        return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: in_type %d / out_type %d", name, in_type,
                    out_type);
    if (act < CBX_ACT_NONE || act > CBX_ACT_GELU_TANH)
        return fail(CBX_ERR_INVALID_ARG, "%s: act %d", name, act);
    if (n_rows == 0) return ok();
    if (!x || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL x or y", name);

    LnArgs a{x, r, in_stride, g, b, eps, n_rows, (int)H, s, y, out_stride, mask};
    const int V = in_type == CBX_TYPE_F32 ? 4 : 8;
    const int in_sz = type_size(in_type), out_sz = type_size(out_type);
    bool vec_ok = (H % V) == 0 && aligned16(x) && (!r || aligned16(r)) && (!s || aligned16(s)) &&
                  aligned16(y) && (!g || aligned16(g)) && (!b || aligned16(b)) &&
                  (in_stride * in_sz) % 16 == 0 && (!s || (out_stride * in_sz) % 16 == 0) &&
                  (out_stride * out_sz) % 16 == 0 && (H / V + 31) / 32 <= 16;
    switch (in_type) {
        case CBX_TYPE_F32: return dispatch_out<float>(a, out_type, act, vec_ok, st, name);
        case CBX_TYPE_BF16: return dispatch_out<__nv_bfloat16>(a, out_type, act, vec_ok, st, name);
        default: return dispatch_out<__half>(a, out_type, act, vec_ok, st, name);
    }
}

}  // namespace cbx

extern "C" CBX_API int cbx_add_layernorm(const void* x, const void* resid, int in_type,
                                         int64_t in_row_stride, const float* gamma,
                                         const float* beta, float eps, int64_t n_rows,
                                         int64_t hidden, void* sum_out, void* y, int out_type,
                                         int64_t out_row_stride, cbx_stream_t stream) {
    return cbx::row_layernorm(x, resid, in_type, in_row_stride, gamma, beta, eps, n_rows, hidden,
                              sum_out, y, out_type, out_row_stride, CBX_ACT_NONE, nullptr,
                              reinterpret_cast<cudaStream_t>(stream), "cbx_add_layernorm");
}
