// k_ln_channels.cu — CFM CausalBlock1D tail: LayerNorm over the channel axis
// of a channels-first [B][C][T] tensor, fused activation (Mish) and mask.
//
// Tile = one batch item x 32 consecutive time steps x all C channels.  Eight
// warps split the channels; lane l owns time step t0 + l, so every shared-
// memory read and every global store of a warp is 32 consecutive floats of one
// channel row (one 128-byte line).  Per-column sums cross the warps through
// shared memory (mean, then squared deviations).  The tensor is read once and
// written once: 8 bytes per element of HBM traffic.
//
// Main path (k_ln_bct_tma): persistent CTAs; each tile [C][16] is staged into
// shared memory by one TMA bulk tensor copy (cp.async.bulk.tensor.3d, no
// multicast) into a 2-deep ring, so the copy of the next tile is in
// flight while the current one is normalised.  Fallbacks: the register-tile
// kernel k_ln_bct (T % 4 != 0, C > 256, unaligned x) and a per-column kernel
// for C > 256 or C % 8 != 0.
//
// cbx_causal_block1d_tail (the causal conv's epilogue + the block tail:
// conv bias, [B][C][T] -> [B][T][C], LN over C, act, mask) is the TAIL
// instance of k_ln_bct_tma: outputs staged in a 128-byte
// swizzled tile and written by TMA tensor stores.
//
// The engine-native [B][T][C] layout is the row-wise kernel in k_layernorm.cu.
#include <cuda.h>  // CUtensorMap and its enums; the encoder is fetched at run time
#include <math.h>
#include <stdlib.h>

#include <map>
#include <mutex>

#include "cbx_common.cuh"

namespace cbx {

int row_layernorm(const void* x, const void* r, int in_type, int64_t in_stride, const float* g,
                  const float* b, float eps, int64_t n_rows, int64_t H, void* s, void* y,
                  int out_type, int64_t out_stride, int act, const float* mask, cudaStream_t st,
                  const char* name);

namespace {

constexpr int kWarps = 8;
constexpr int kCols = 32;

// CBX_LN_CHANNELS_NO_TMA=1 selects the register-tile kernel even where the
// TMA kernel applies (A/B measurements).
bool force_register_path() {
    static const bool v = [] {
        const char* e = getenv("CBX_LN_CHANNELS_NO_TMA");
        return e && e[0] && e[0] != '0';
    }();
    return v;
}

// CBX_LN_CHANNELS_GENERIC=1 selects the per-column kernel for any shape (A/B
// measurements and profiles of the fallback).
bool force_generic_path() {
    static const bool v = [] {
        const char* e = getenv("CBX_LN_CHANNELS_GENERIC");
        return e && e[0] && e[0] != '0';
    }();
    return v;
}

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
    const float* cb;  // conv bias added before the statistics (causal block tail), or NULL
    bool out_btc;     // y in [B][T][C] (causal block tail) instead of x's [B][C][T]
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

// Device error word of this library: bit CBX_DEVERR_WAIT_TIMEOUT is set by a
// bounded wait that gave up (read and cleared by cbx_device_errors).
__device__ int g_device_errors;

// Ring depth of the TMA kernel: 2 stages (32 KB at C = 256) for both
// instances.  With 4 CTAs per SM that keeps 8 tiles in flight per SM and
// leaves shared memory free for the next kernel's CTAs to become resident
// early under PDL; the tail's output staging fits beside it.  Measured at
// [32,256,1000] in config 3's step (LN over C + Mish, then the timestep
// embedding): 3 stages 15.11 us per step (LN 14.56 us), 2 stages 14.31 us
// (LN 14.33 us); 2 stages at 5 CTAs per SM (48 registers) 14.65 us.
constexpr int kStages = 2;
template <bool TAIL> constexpr int ring_stages() { return kStages; }
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// TMA tensor store of a shared-memory box (no multicast), tracked as a bulk
// async-group of the issuing thread.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y,
                                             int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(z), "r"(smem_addr(src))
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The committed stores have finished reading shared memory / have completed.
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Diagnostic for the bounded-wait path: one thread initialises an mbarrier
// that nothing will ever complete (no copy is issued), waits on it for at
// most `polls` polls exactly as the TMA kernels do, and on expiry raises
// CBX_DEVERR_WAIT_TIMEOUT in the device error word.
__global__ void k_selftest_wait(uint32_t polls) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    mbar_fence_init();
    bool done = false;
    for (uint32_t i = 0; i < polls && !done; ++i) done = mbar_try_wait(&bar, 0);
    if (!done) atomicOr(&g_device_errors, CBX_DEVERR_WAIT_TIMEOUT);
}

// TMA tiles are 16 time steps wide: 256 threads = 16 columns x 16 channel
// groups; thread (col, grp) owns channels grp + 16 i (i < CPT, C = 16 CPT).
// The two half-warps of a warp read adjacent channel rows of the tile (64 B
// apart: disjoint banks) and store two 64-byte row segments.  Narrow tiles
// keep the per-CTA tile count balanced on 148 SMs (T = 1000: 63 tiles per
// item).
constexpr int kTCols = 16;
constexpr int kGroups = 256 / kTCols;

// Shared memory: [kStages][C][kTCols] f32 ring filled by TMA.
// TAIL (the causal block tail): conv bias added to each value before the
// statistics, and the outputs written as [B][T][C] by TMA tensor stores
// (ymap: dims (C, T, B), box 32 channels x kTCols steps, 128-byte swizzle).
// The tile is staged as C / 32 chunks of [kTCols][32] f32 in the swizzled
// layout (16-byte unit u of row r at unit u ^ (r % 8)), so a warp's 32
// staging writes fall in 16 distinct 4-bank groups; rows past T are clipped by
// the store.
template <int CPT, int ACT, bool TAIL>
__global__ void __launch_bounds__(256, 4) k_ln_bct_tma(const __grid_constant__ CUtensorMap tmap,
                                                       const __grid_constant__ CUtensorMap ymap,
                                                       ChArgs a) {
    constexpr int C = kGroups * CPT;
    constexpr int kTileElems = C * kTCols;
    constexpr uint32_t kTileBytes = kTileElems * 4u;
    constexpr int NS = ring_stages<TAIL>();
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ float2 affine[C];  // (gamma, beta) per channel
    __shared__ uint64_t bars[NS];
    __shared__ float2 part[2][kWarps][kTCols];  // per-warp (mean, M2) of each column
    float* tiles = reinterpret_cast<float*>(smem);
    // TAIL staging: [C / 32][kTCols][32] f32, 1024-byte aligned (after the ring)
    unsigned char* ostage = smem + (size_t)NS * kTileBytes;

    const int col = threadIdx.x % kTCols;
    const int grp = threadIdx.x / kTCols;
    // tiles of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
    const int64_t mine =
        a.n_tiles > blockIdx.x ? (a.n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    if constexpr (TAIL) {
        // the 128-byte swizzle is defined on 1024-byte aligned shared memory:
        // refuse (before any copy is issued) rather than scramble the output
        if (smem_addr(ostage) & 1023u) {
            if (threadIdx.x == 0) atomicOr(&g_device_errors, CBX_DEVERR_SMEM_ALIGN);
            return;
        }
    }

    if (threadIdx.x == 0) {
        for (int st = 0; st < NS; ++st) mbar_init(&bars[st], 1);
        mbar_fence_init();
    }
    grid_dep_wait();
    grid_dep_launch();
    auto issue = [&](int64_t k) {  // thread 0: TMA of this CTA's k-th tile into its stage
        const int tile = (int)(blockIdx.x + k * gridDim.x);
        const int bi = tile / a.tiles_per_item;
        const int t0 = (tile - bi * a.tiles_per_item) * kTCols;
        const int st = (int)(k % NS);
        mbar_arrive_expect_tx(&bars[st], kTileBytes);
        tma_load_3d(tiles + st * kTileElems, &tmap, t0, 0, bi, &bars[st]);
    };
    if (threadIdx.x == 0)
        for (int64_t k = 0; k < mine && k < NS; ++k) issue(k);
    for (int c = threadIdx.x; c < C; c += blockDim.x)
        affine[c] = make_float2(a.g ? a.g[c] : 1.0f, a.b ? a.b[c] : 0.0f);
    // TAIL: the conv bias of this thread's channels (fixed across tiles) in registers
    float cbr[TAIL ? CPT : 1];
#pragma unroll
    for (int i = 0; i < (TAIL ? CPT : 1); ++i)
        cbr[i] = (TAIL && a.cb) ? __ldg(a.cb + grp + kGroups * i) : 0.0f;
    // Every thread polls the ring's mbarriers below, and polling one before
    // thread 0's mbarrier.init is undefined: this barrier orders the inits
    // (and the affine table) before any wait or read.
    __syncthreads();
    constexpr float kInvCpt = 1.0f / (float)CPT;
    constexpr float kInvC = 1.0f / (float)C;
    // (item, tile-in-item) of this CTA's k-th tile, advanced without a division
    const int step_bi = (int)(gridDim.x / a.tiles_per_item);
    const int step_tl = (int)(gridDim.x - step_bi * a.tiles_per_item);
    int cur_bi = (int)(blockIdx.x / a.tiles_per_item);
    int cur_tl = (int)(blockIdx.x - cur_bi * a.tiles_per_item);
    const bool has_mask = a.mask != nullptr;
    const int64_t cstride = (int64_t)kGroups * a.T;  // between a thread's channels in y

    for (int64_t k = 0; k < mine; ++k) {
        const int st = (int)(k % NS);
        const uint32_t parity = (uint32_t)((k / NS) & 1);
        // every thread waits (bounded) for the tile; the barrier below turns
        // the outcome into one CTA-wide decision
        const bool ok = mbar_wait_bounded(&bars[st], parity);
        const float* tl = tiles + st * kTileElems + grp * kTCols + col;
        float v[CPT];
        // (after a failed wait the values are stale shared memory; every thread
        // then leaves at the barrier below without using them)
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            v[i] = tl[i * kGroups * kTCols];
            if constexpr (TAIL) v[i] = __fadd_rn(v[i], cbr[i]);  // ggml_add
        }
        // sum and squared deviations over channel pairs on packed f32x2 (CPT is even)
        float2 s2 = make_float2(v[0], v[1]);
#pragma unroll
        for (int i = 2; i < CPT; i += 2) s2 = __fadd2_rn(s2, make_float2(v[i], v[i + 1]));
        float m = (s2.x + s2.y) * kInvCpt;
        float2 q2 = pair(0.0f);
#pragma unroll
        for (int i = 0; i < CPT; i += 2) {
            const float2 d = __fadd2_rn(make_float2(v[i], v[i + 1]), pair(-m));
            q2 = __ffma2_rn(d, d, q2);
        }
        float q = q2.x + q2.y;
        // the warp's two groups (lanes l and l ^ 16 share a column): merge by
        // shuffle into (mean, M2) over 2 CPT values
        {
            const float mo = __shfl_xor_sync(0xffffffffu, m, 16);
            const float qo = __shfl_xor_sync(0xffffffffu, q, 16);
            const float d = mo - m;
            q = q + qo + 0.5f * (float)CPT * d * d;
            m = 0.5f * (m + mo);
        }
        // part[] alternates by tile: the next tile writes the other half while
        // slower threads may still read this one
        float2(*pk)[kTCols] = part[k & 1];
        if ((threadIdx.x & 16) == 0) pk[threadIdx.x >> 5][col] = make_float2(m, q);
        if constexpr (TAIL)
            if (threadIdx.x == 0) bulk_wait_read_all();  // previous tile's stores are out of ostage
        if (__syncthreads_or(ok ? 0 : 1)) {
            // A transfer never completed: flag it, give the copies still in
            // flight a bounded chance to land in this CTA's shared memory,
            // and leave (every thread takes this branch together).
            if (threadIdx.x == 0) {
                if constexpr (TAIL) bulk_wait_all();
                atomicOr(&g_device_errors, CBX_DEVERR_WAIT_TIMEOUT);
                for (int64_t j = k + 1; j < mine && j < k + NS; ++j)
                    mbar_wait_bounded(&bars[j % NS], (uint32_t)((j / NS) & 1));
            }
            return;
        }
        // every thread holds its tile values: refill the stage with tile k + NS
        if (threadIdx.x == 0 && k + NS < mine) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(k + NS);
        }
        // merge the warps' partials (equal counts of 2 CPT):
        // mean = avg of means, M2 = sum M2_w + 2 CPT * sum (mean_w - mean)^2
        float mean = 0.0f;
#pragma unroll
        for (int g = 0; g < kWarps; ++g) mean += pk[g][col].x;
        mean *= 1.0f / (float)kWarps;
        float m2 = 0.0f, dm = 0.0f;
#pragma unroll
        for (int g = 0; g < kWarps; ++g) {
            const float2 pq = pk[g][col];
            m2 += pq.y;
            const float d = pq.x - mean;
            dm = fmaf(d, d, dm);
        }
        m2 = fmaf(2.0f * (float)CPT, dm, m2);
        const float rstd = rsqrtf(m2 * kInvC + a.eps);

        const int bi = cur_bi;
        const int t0 = cur_tl * kTCols;
        const int t = t0 + col;
        cur_tl += step_tl;
        cur_bi += step_bi;
        if (cur_tl >= a.tiles_per_item) {
            cur_tl -= a.tiles_per_item;
            ++cur_bi;
        }
        if constexpr (TAIL) {
            const float mk = (has_mask && t < a.T) ? a.mask[(int64_t)bi * a.T + t] : 1.0f;
#pragma unroll
            for (int i = 0; i < CPT; i += 2) {
                // channels ch and ch + kGroups on packed pairs
                const int ch = grp + kGroups * i;
                const float2 g0 = affine[ch], g1 = affine[ch + kGroups];
                float2 o = __ffma2_rn(
                    __fmul2_rn(__fadd2_rn(make_float2(v[i], v[i + 1]), pair(-mean)), pair(rstd)),
                    make_float2(g0.x, g1.x), make_float2(g0.y, g1.y));
                if constexpr (ACT != CBX_ACT_NONE) o = act_f2<ACT>(o);
                if (has_mask) o = __fmul2_rn(o, pair(mk));
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c2 = ch + h * kGroups;
                    const int cc = c2 & 31;
                    const uint32_t off = (uint32_t)(c2 >> 5) * (kTCols * 128u) + (uint32_t)col * 128u +
                                         ((uint32_t)((cc >> 2) ^ (col & 7)) << 4) + (uint32_t)(cc & 3) * 4u;
                    *reinterpret_cast<float*>(ostage + off) = h ? o.y : o.x;
                }
            }
            fence_async_shared();  // this thread's staging writes before the TMA store reads them
            __syncthreads();
            if (threadIdx.x == 0) {
#pragma unroll
                for (int q = 0; q < C / 32; ++q)
                    tma_store_3d(&ymap, ostage + q * (kTCols * 128), q * 32, t0, bi);
                bulk_commit();
            }
            // thread 0 waits for the stores' shared-memory reads before the
            // next tile's first barrier, after which ostage is rewritten
        } else if (t < a.T) {
            const float mk = has_mask ? a.mask[(int64_t)bi * a.T + t] : 1.0f;
            float* yc = a.y + ((int64_t)bi * C + grp) * a.T + t;
#pragma unroll
            for (int i = 0; i < CPT; i += 2) {
                // channels grp + kGroups i and the next on packed pairs
                const float2 g0 = affine[grp + kGroups * i], g1 = affine[grp + kGroups * (i + 1)];
                float2 o = __ffma2_rn(
                    __fmul2_rn(__fadd2_rn(make_float2(v[i], v[i + 1]), pair(-mean)), pair(rstd)),
                    make_float2(g0.x, g1.x), make_float2(g0.y, g1.y));
                if constexpr (ACT != CBX_ACT_NONE) o = act_f2<ACT>(o);
                if (has_mask) o = __fmul2_rn(o, pair(mk));
                yc[0] = o.x;
                yc[cstride] = o.y;
                yc += 2 * cstride;
            }
        }
        // part[k & 1] is rewritten by tile k + 2, after tile k + 1's barrier,
        // which every thread reaches only after its reads above.
    }
    if constexpr (TAIL)
        if (threadIdx.x == 0) bulk_wait_all();  // the last tile's stores have completed
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
        // conv bias (causal block tail) rounded in f32 as ggml_add
        auto val = [&](int c) {
            const float v = xc[(int64_t)c * a.T];
            return a.cb ? __fadd_rn(v, a.cb[c]) : v;
        };
        float s = 0.0f;
        for (int c = 0; c < a.C; ++c) s += val(c);
        const float mean = s / (float)a.C;
        float q = 0.0f;
        for (int c = 0; c < a.C; ++c) {
            const float d = val(c) - mean;
            q = fmaf(d, d, q);
        }
        const float rstd = 1.0f / sqrtf(q / (float)a.C + a.eps);
        const float m = a.mask ? a.mask[bi * a.T + t] : 1.0f;
        float* yc = a.out_btc ? a.y + (bi * a.T + t) * a.C : a.y + bi * a.C * a.T + t;
        const int64_t ystride = a.out_btc ? 1 : a.T;
        for (int c = 0; c < a.C; ++c) {
            float o = fmaf((val(c) - mean) * rstd, a.g ? a.g[c] : 1.0f, a.b ? a.b[c] : 0.0f);
            if constexpr (ACT != CBX_ACT_NONE) o = act_f<ACT>(o);
            yc[(int64_t)c * ystride] = o * m;
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

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// TMA path conditions: x 16-byte aligned, T * 4 a multiple of 16 (row
// stride), T >= 16, C in {32, 64, 128, 256} (one box spans all channels, 16
// groups of C / 16).
bool tma_ok(const ChArgs& a) {
    return aligned16(a.x) && (a.T % 4) == 0 && a.T >= kTCols &&
           (int64_t)a.B * ((a.T + kTCols - 1) / kTCols) < ((int64_t)1 << 31) &&
           (a.C == 32 || a.C == 64 || a.C == 128 || a.C == 256) &&
           (int64_t)a.C * a.T < ((int64_t)1 << 31) && encoder() != nullptr;
}

template <int CPT, int ACT, bool TAIL>
int launch_bct_tma(const ChArgs& a, cudaStream_t st) {
    constexpr int C = kGroups * CPT;
    CUtensorMap map;
    cuuint64_t dims[3] = {(cuuint64_t)a.T, (cuuint64_t)C, (cuuint64_t)a.B};
    cuuint64_t strides[2] = {(cuuint64_t)a.T * 4, (cuuint64_t)C * a.T * 4};
    cuuint32_t box[3] = {(cuuint32_t)kTCols, (cuuint32_t)C, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(a.x), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(CBX_ERR_CUDA, "cbx_layernorm_channels: cuTensorMapEncodeTiled failed (%d)",
                    (int)r);
    CUtensorMap ymap = map;  // unused unless TAIL
    if (TAIL) {
        cuuint64_t ydims[3] = {(cuuint64_t)C, (cuuint64_t)a.T, (cuuint64_t)a.B};
        cuuint64_t ystrides[2] = {(cuuint64_t)C * 4, (cuuint64_t)C * a.T * 4};
        cuuint32_t ybox[3] = {32, (cuuint32_t)kTCols, 1};
        r = encoder()(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.y, ydims, ystrides, ybox, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(CBX_ERR_CUDA, "cbx_causal_block1d_tail: cuTensorMapEncodeTiled (y) failed (%d)",
                        (int)r);
    }
    auto kern = k_ln_bct_tma<CPT, ACT, TAIL>;
    constexpr size_t smem =
        (size_t)ring_stages<TAIL>() * C * kTCols * 4 + (TAIL ? (size_t)kTCols * C * 4 : 0);
    if (!smem_opt_in(kern, smem)) return fail(CBX_ERR_CUDA, "cbx_layernorm_channels: shared memory opt-in failed");
    const int occ = occupancy(kern, 256, smem);
    // CTAs per SM: as many as fit.  Measured at [32,256,1000] (2016 tiles),
    // in a step that alternates this kernel with another: 4 per SM 15.8 us per
    // step, 3 per SM (an even 4.5 tiles per CTA) 16.8 us, 2 per SM 17.1 us.
    const int sms = num_sms();
    const int per_sm = occ;
    int64_t blocks = (int64_t)sms * per_sm;
    if (blocks > a.n_tiles) blocks = a.n_tiles;
    return launch_status(launch(kern, dim3((unsigned)blocks), dim3(256), smem, st, map, ymap, a),
                         TAIL ? "cbx_causal_block1d_tail" : "cbx_layernorm_channels");
}

template <int ACT, bool TAIL>
int dispatch_tma(const ChArgs& a, cudaStream_t st) {
    ChArgs t = a;  // TMA tiles are kTCols wide
    t.tiles_per_item = (a.T + kTCols - 1) / kTCols;
    t.n_tiles = (int64_t)a.B * t.tiles_per_item;
    switch (a.C) {
        case 32: return launch_bct_tma<2, ACT, TAIL>(t, st);
        case 64: return launch_bct_tma<4, ACT, TAIL>(t, st);
        case 128: return launch_bct_tma<8, ACT, TAIL>(t, st);
        default: return launch_bct_tma<16, ACT, TAIL>(t, st);
    }
}

template <int ACT>
int launch_generic(const ChArgs& a, cudaStream_t st, const char* name) {
    auto kern = k_ln_bct_generic<ACT>;
    const int64_t ncol = (int64_t)a.B * a.T;
    int64_t blocks = (ncol + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    return launch_status(launch(kern, dim3((unsigned)blocks), dim3(256), 0, st, a), name);
}

template <int ACT>
int dispatch_bct(const ChArgs& a, cudaStream_t st) {
    const int cpw = a.C / kWarps;
    if (force_generic_path())
        return launch_generic<ACT>(a, st, a.out_btc ? "cbx_causal_block1d_tail" : "cbx_layernorm_channels");
    if (a.out_btc) {  // causal block tail: TMA kernel, else one thread per column
        if (tma_ok(a) && aligned16(a.y) && !force_register_path())
            return dispatch_tma<ACT, true>(a, st);
        return launch_generic<ACT>(a, st, "cbx_causal_block1d_tail");
    }
    if (tma_ok(a) && !force_register_path()) return dispatch_tma<ACT, false>(a, st);
    const bool fits = (a.C % kWarps) == 0 && (int64_t)a.C * a.T < ((int64_t)1 << 31);
    if (fits && cpw <= 8) return launch_bct<8, ACT>(a, st);
    if (fits && cpw <= 16) return launch_bct<16, ACT>(a, st);
    if (fits && cpw <= 32) return launch_bct<32, ACT>(a, st);
    return launch_generic<ACT>(a, st, "cbx_layernorm_channels");
}

}  // namespace

// Looked up on every call (it is cheap next to a launch), so the address is
// always the current device's and current context's.
int* device_error_word() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_errors) != cudaSuccess) return nullptr;
    return static_cast<int*>(p);
}

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
    a.cb = nullptr;
    a.out_btc = false;
    switch (act) {
        case CBX_ACT_MISH: return dispatch_bct<CBX_ACT_MISH>(a, st);
        case CBX_ACT_SILU: return dispatch_bct<CBX_ACT_SILU>(a, st);
        case CBX_ACT_GELU_TANH: return dispatch_bct<CBX_ACT_GELU_TANH>(a, st);
        default: return dispatch_bct<CBX_ACT_NONE>(a, st);
    }
}

// cfm_decoder.cpp:114-115 (conv bias, transpose back to (C, T)) and
// :144-148 (LN over C, Mish, mask) after the causal conv's GEMM.
extern "C" CBX_API int cbx_causal_block1d_tail(const float* x, const float* conv_bias,
                                               const float* gamma, const float* beta, float eps,
                                               const float* mask, int64_t B, int64_t C,
                                               int64_t T, int act, float* y,
                                               cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_causal_block1d_tail";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B < 0 || C <= 0 || T < 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: B %lld C %lld T %lld", name, (long long)B,
                    (long long)C, (long long)T);
    if (act < CBX_ACT_NONE || act > CBX_ACT_GELU_TANH)
        return fail(CBX_ERR_INVALID_ARG, "%s: act %d", name, act);
    if (!(eps >= 0.0f)) return fail(CBX_ERR_INVALID_ARG, "%s: eps must be >= 0", name);
    if (B > INT32_MAX || C > INT32_MAX || T > INT32_MAX)
        return fail(CBX_ERR_INVALID_ARG, "%s: dimension exceeds 2^31-1", name);
    if (B == 0 || T == 0) return ok();
    if (!x || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL x or y", name);
    if (x == y) return fail(CBX_ERR_INVALID_ARG, "%s: y must not alias x (layouts differ)", name);
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
    a.cb = conv_bias;
    a.out_btc = true;
    switch (act) {
        case CBX_ACT_MISH: return dispatch_bct<CBX_ACT_MISH>(a, st);
        case CBX_ACT_SILU: return dispatch_bct<CBX_ACT_SILU>(a, st);
        case CBX_ACT_GELU_TANH: return dispatch_bct<CBX_ACT_GELU_TANH>(a, st);
        default: return dispatch_bct<CBX_ACT_NONE>(a, st);
    }
}

extern "C" CBX_API int cbx_device_errors(int32_t* flags, cbx_stream_t stream) {
    using namespace cbx;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t v = 0;
    const int32_t zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_device_errors, sizeof(v), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbolAsync(g_device_errors, &zero, sizeof(zero), 0,
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return fail(CBX_ERR_CUDA, "cbx_device_errors: %s", cudaGetErrorString(e));
    if (flags) *flags = v;
    if (v) return fail(CBX_ERR_TIMEOUT, "cbx_device_errors: device error bits 0x%x", v);
    return ok();
}

extern "C" CBX_API int cbx_selftest_wait_timeout(uint32_t polls, cbx_stream_t stream) {
    using namespace cbx;
    if (polls == 0 || polls > kMaxPolls)
        return fail(CBX_ERR_INVALID_ARG, "cbx_selftest_wait_timeout: polls must be in [1, 2^24]");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    k_selftest_wait<<<1, 32, 0, st>>>(polls);
    return launch_status(cudaGetLastError(), "cbx_selftest_wait_timeout");
}
