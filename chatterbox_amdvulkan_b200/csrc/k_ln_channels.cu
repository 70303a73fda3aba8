// k_ln_channels.cu — CFM CausalBlock1D tail: LayerNorm over the channel axis
// of a channels-first [B][C][T] tensor, fused activation (Mish) and mask.
//
// Tile = one batch item x 32 consecutive time steps x all C channels.  Eight
// warps split the channels; lane l owns time step t0 + l, so every warp load
// or store is 32 consecutive floats (one 128-byte line) of one channel row.
// Each thread keeps its channel values in registers; per-column sums cross the
// warps through 1 KB of shared memory (mean, then squared deviations).  The
// tensor is read once and written once: 8 bytes per element of HBM traffic.
//
// The engine-native [B][T][C] layout is the row-wise kernel in k_layernorm.cu.
#include "cbx_common.cuh"

namespace cbx {

int row_layernorm(const void* x, const void* r, int in_type, int64_t in_stride, const float* g,
                  const float* b, float eps, int64_t n_rows, int64_t H, void* s, void* y,
                  int out_type, int64_t out_stride, int act, const float* mask, cudaStream_t st,
                  const char* name);

namespace {

constexpr int kWarps = 8;
constexpr int kCols = 32;

struct ChArgs {
    const float* x;
    const float* g;
    const float* b;
    float eps;
    const float* mask;
    int B, C, T;
    int tiles_per_item;
    int64_t n_tiles;
    float* y;
};

// MAXC = channels held per warp (>= C / kWarps; C % kWarps == 0).  gamma and
// beta are staged in shared memory once per CTA; offsets within a batch item
// are 32-bit (C * T < 2^31 is checked on the host).
template <int MAXC, int ACT>
__global__ void __launch_bounds__(kWarps * 32, 2) k_ln_bct(ChArgs a) {
    extern __shared__ float gb[];  // [2][C]
    __shared__ float red[kWarps][kCols];
    __shared__ float stat[2][kCols];
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    const int cpw = a.C / kWarps;
    const int c0 = w * cpw;
    const float inv_c = 1.0f / (float)a.C;
    for (int c = threadIdx.x; c < a.C; c += blockDim.x) {
        gb[c] = a.g ? a.g[c] : 1.0f;
        gb[a.C + c] = a.b ? a.b[c] : 0.0f;
    }
    // the first tile's barrier orders these writes before any read

    for (int64_t tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
        const int bi = (int)(tile / a.tiles_per_item);
        const int t = (int)(tile - (int64_t)bi * a.tiles_per_item) * kCols + lane;
        const bool tv = t < a.T;
        const int64_t item = (int64_t)bi * a.C * a.T;
        const float* xb = a.x + item + t;
        float v[MAXC];
        int off = c0 * a.T;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            v[i] = (tv && i < cpw) ? xb[off] : 0.0f;
            off += a.T;
        }
        float p = 0.0f;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) p += v[i];
        red[w][lane] = p;
        __syncthreads();
        if (w == 0) {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < kWarps; ++k) s += red[k][lane];
            stat[0][lane] = s * inv_c;
        }
        __syncthreads();
        const float mean = stat[0][lane];
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            if (i < cpw) {
                const float d = v[i] - mean;
                q = fmaf(d, d, q);
            }
        }
        red[w][lane] = q;
        __syncthreads();
        if (w == 0) {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < kWarps; ++k) s += red[k][lane];
            stat[1][lane] = 1.0f / sqrtf(s * inv_c + a.eps);
        }
        __syncthreads();
        const float rstd = stat[1][lane];
        const float m = (a.mask && tv) ? a.mask[(int64_t)bi * a.T + t] : 1.0f;
        float* yb = a.y + item + t;
        off = c0 * a.T;
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            if (tv && i < cpw) {
                float o = fmaf((v[i] - mean) * rstd, gb[c0 + i], gb[a.C + c0 + i]);
                if constexpr (ACT != CBX_ACT_NONE) o = act_f<ACT>(o);
                yb[off] = o * m;
            }
            off += a.T;
        }
        // red/stat are rewritten by the next tile only after its first barrier
    }
}

// Any C: one thread per (b, t) column, three passes over the column (the
// re-reads are served by L1/L2).
template <int ACT>
__global__ void __launch_bounds__(256) k_ln_bct_generic(ChArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t ncol = (int64_t)a.B * a.T;
    for (int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; col < ncol;
         col += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bi = col / a.T, t = col - bi * a.T;
        const float* xc = a.x + bi * a.C * a.T + t;
        float s = 0.0f;
        for (int c = 0; c < a.C; ++c) s += xc[(int64_t)c * a.T];
        const float mean = s / (float)a.C;
        float q = 0.0f;
        for (int c = 0; c < a.C; ++c) {
            const float d = xc[(int64_t)c * a.T] - mean;
            q = fmaf(d, d, q);
        }
        const float rstd = 1.0f / sqrtf(q / (float)a.C + a.eps);
        const float m = a.mask ? a.mask[bi * a.T + t] : 1.0f;
        float* yc = a.y + bi * a.C * a.T + t;
        for (int c = 0; c < a.C; ++c) {
            float o = fmaf((xc[(int64_t)c * a.T] - mean) * rstd, a.g ? a.g[c] : 1.0f,
                           a.b ? a.b[c] : 0.0f);
            if constexpr (ACT != CBX_ACT_NONE) o = act_f<ACT>(o);
            yc[(int64_t)c * a.T] = o * m;
        }
    }
}

template <int MAXC, int ACT>
int launch_bct(const ChArgs& a, cudaStream_t st) {
    auto kern = k_ln_bct<MAXC, ACT>;
    const size_t smem = 2 * (size_t)a.C * sizeof(float);
    const int occ = occupancy(kern, kWarps * 32, smem);
    int64_t blocks = a.n_tiles;
    const int64_t cap = (int64_t)num_sms() * occ;
    if (blocks > cap) blocks = cap;
    return launch_status(launch(kern, dim3((unsigned)blocks), dim3(kWarps * 32), smem, st, a),
                         "cbx_layernorm_channels");
}

template <int ACT>
int dispatch_bct(const ChArgs& a, cudaStream_t st) {
    const int cpw = a.C / kWarps;
    const bool fits = (a.C % kWarps) == 0 && (int64_t)a.C * a.T < ((int64_t)1 << 31);
    if (fits && cpw <= 8) return launch_bct<8, ACT>(a, st);
    if (fits && cpw <= 16) return launch_bct<16, ACT>(a, st);
    if (fits && cpw <= 32) return launch_bct<32, ACT>(a, st);
    auto kern = k_ln_bct_generic<ACT>;
    const int64_t ncol = (int64_t)a.B * a.T;
    int64_t blocks = (ncol + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    return launch_status(launch(kern, dim3((unsigned)blocks), dim3(256), 0, st, a),
                         "cbx_layernorm_channels");
}

}  // namespace
}  // namespace cbx

extern "C" CBX_API int cbx_layernorm_channels(const float* x, const float* gamma,
                                              const float* beta, float eps, const float* mask,
                                              int64_t B, int64_t C, int64_t T, int layout,
                                              int act, float* y, cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_layernorm_channels";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B < 0 || C <= 0 || T < 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: B %lld C %lld T %lld", name, (long long)B,
                    (long long)C, (long long)T);
    if (layout != CBX_LAYOUT_BCT && layout != CBX_LAYOUT_BTC)
        return fail(CBX_ERR_INVALID_ARG, "%s: layout %d", name, layout);
    if (act < CBX_ACT_NONE || act > CBX_ACT_GELU_TANH)
        return fail(CBX_ERR_INVALID_ARG, "%s: act %d", name, act);
    if (!(eps >= 0.0f)) return fail(CBX_ERR_INVALID_ARG, "%s: eps must be >= 0", name);
    if (B > INT32_MAX || C > INT32_MAX || T > INT32_MAX)
        return fail(CBX_ERR_INVALID_ARG, "%s: dimension exceeds 2^31-1", name);
    if (B == 0 || T == 0) return ok();
    if (!x || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL x or y", name);
    if (layout == CBX_LAYOUT_BTC)
        return row_layernorm(x, nullptr, CBX_TYPE_F32, C, gamma, beta, eps, B * T, C, nullptr, y,
                             CBX_TYPE_F32, C, act, mask, st, name);
    ChArgs a;
    a.x = x;
    a.g = gamma;
    a.b = beta;
    a.eps = eps;
    a.mask = mask;
    a.B = (int)B;
    a.C = (int)C;
    a.T = (int)T;
    a.tiles_per_item = (int)((T + kCols - 1) / kCols);
    a.n_tiles = B * (int64_t)a.tiles_per_item;
    a.y = y;
    switch (act) {
        case CBX_ACT_MISH: return dispatch_bct<CBX_ACT_MISH>(a, st);
        case CBX_ACT_SILU: return dispatch_bct<CBX_ACT_SILU>(a, st);
        case CBX_ACT_GELU_TANH: return dispatch_bct<CBX_ACT_GELU_TANH>(a, st);
        default: return dispatch_bct<CBX_ACT_NONE>(a, st);
    }
}
