// k_embed.cu — token + learned-position embedding gather-add, and the T3
// prefill sequence [cond rows ; speech_emb[prompt] ; tok_table[tokens]] + pos.
//
// The output rows are split into contiguous blocks, one per warp (the CTA's
// warps own one contiguous range, whose ids are prefetched into L2 before the
// PDL wait).  A warp walks its rows in groups of 32: each lane loads one row's
// id and position (one coalesced load per 32 rows, so no row waits on its own
// id load), and the warp then takes the group's rows two at a time, with the
// ids broadcast by shuffle.  For a pair of rows every lane issues all of its
// table loads (4 16-byte vectors of each row from each table) before any add,
// 16 loads in flight per lane.  Rows are widened to f32, added once and
// rounded once to the output type; stores are 16-byte vectors, coalesced.
//
// Compulsory HBM traffic: the output, the ids and every distinct table row
// once.  The speech table (6563 x 1024) and the position table stay in L2
// across rows; the 50276 x 1024 text table (103 MB in f16) does not, so its
// distinct rows come from HBM.
#include <type_traits>

#include "cbx_common.cuh"

namespace cbx {
namespace {

constexpr int kPer = 4;   // 16-byte vectors per lane per row and pass
constexpr int kWarps = 8; // warps per CTA of the vector kernel

// Rows [0, n_cond) copy f32 rows of `cond`; rows [n_cond, seg1_end) gather
// seg1.table[seg1.ids[r - n_cond]]; rows [seg1_end, n_rows) gather
// seg2.table[seg2.ids[r - seg1_end]].  cbx_embed_gather_add is one segment
// (seg2) with n_cond = seg1_end = 0.
struct Seg {
    const void* table;
    int64_t n_rows;
    const int32_t* ids;
};

struct EmbArgs {
    const float* cond;
    int64_t n_cond;
    Seg seg1;
    int64_t seg1_end;
    Seg seg2;
    const void* pos;
    int64_t n_pos;
    const int32_t* pos_ids;
    int64_t pos_offset;
    int64_t pos_period;  // > 0: position of row r is pos_offset + r % pos_period
    int64_t n_rows;
    int H;
    void* out;
    int32_t* err;
    int64_t rows_per_warp;
    // Batched sequences (cbx_t3_embed_sequence_batched): grid row blockIdx.y
    // is utterance b, whose cond rows, id arrays and output start b times
    // these strides (elements) further on; 0 for single-sequence calls.
    int64_t cond_bstride, seg1_bstride, seg2_bstride, out_bstride;
};

// Points `a` at utterance blockIdx.y of a batched call (strides 0 for one
// sequence).  The conditioning rows' pointer is also formed from the kernel
// argument at its use (cond_of): the copy's cond field did not move for
// utterances b > 0 on the vector path in a GPU test, and forming it at the
// use made every utterance bit-exact.
template <typename TO>
__device__ __forceinline__ void select_item(EmbArgs& a) {
    const int64_t b = blockIdx.y;
    a.cond += b * a.cond_bstride;
    a.seg1.ids += b * a.seg1_bstride;
    a.seg2.ids += b * a.seg2_bstride;
    a.out = static_cast<TO*>(a.out) + b * a.out_bstride;
}
// Conditioning rows of utterance blockIdx.y, from the kernel argument.
__device__ __forceinline__ const float* cond_of(const EmbArgs& args) {
    return args.cond + (int64_t)blockIdx.y * args.cond_bstride;
}

// Segment of row r: 0 cond, 1 seg1, 2 seg2.
__device__ __forceinline__ int seg_of(const EmbArgs& a, int64_t r) {
    return r < a.n_cond ? 0 : (r < a.seg1_end ? 1 : 2);
}

// Row id and position of row r; flags of an out-of-range id / position.
__device__ __forceinline__ void row_source(const EmbArgs& a, int64_t r, int64_t* id, int64_t* p,
                                           int* flags) {
    const int s = seg_of(a, r);
    int64_t i = 0;
    int f = 0;
    if (s == 1) {
        i = a.seg1.ids[r - a.n_cond];
        if (i < 0 || i >= a.seg1.n_rows) f |= CBX_EFLAG_TOKEN_OOB;
    } else if (s == 2) {
        i = a.seg2.ids[r - a.seg1_end];
        if (i < 0 || i >= a.seg2.n_rows) f |= CBX_EFLAG_TOKEN_OOB;
    } else {
        i = r;  // cond row r
    }
    const int64_t q = a.pos_ids      ? (int64_t)a.pos_ids[r]
                      : a.pos_period ? a.pos_offset + r % a.pos_period
                                     : a.pos_offset + r;
    if (a.pos && (q < 0 || q >= a.n_pos)) f |= CBX_EFLAG_POS_OOB;
    *id = i;
    *p = q;
    *flags = f;
}

__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ float load_any(const void* p, int type, int64_t i) {
    if (type == CBX_TYPE_F32) return static_cast<const float*>(p)[i];
    if (type == CBX_TYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// Sum of two 16-byte vectors of 16-bit T, rounded once to T, by the packed
// bf16x2 / f16x2 add (correctly rounded sum of each pair).  Equal to widening
// to f32, adding and rounding once: when the exponents differ by at most 12
// (f16) / 15 (bf16) the f32 sum is exact; beyond that the smaller operand is
// below half an ulp of the larger in T, and both forms return the larger.
template <typename T>
__device__ __forceinline__ uint4 add16x8(const uint4& x, const uint4& y) {
    uint4 r;
    const uint32_t* xs = &x.x;
    const uint32_t* ys = &y.x;
    uint32_t* rs = &r.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            const __nv_bfloat162 s = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(xs + k),
                                             *reinterpret_cast<const __nv_bfloat162*>(ys + k));
            rs[k] = *reinterpret_cast<const uint32_t*>(&s);
        } else {
            const __half2 s = __hadd2(*reinterpret_cast<const __half2*>(xs + k),
                                      *reinterpret_cast<const __half2*>(ys + k));
            rs[k] = *reinterpret_cast<const uint32_t*>(&s);
        }
    }
    return r;
}

// Widen one 16-byte vector of T to f32.
template <typename T>
__device__ __forceinline__ void widen(const uint4& w, float (&f)[Vec<T>::n]) {
    constexpr int k = 4 / (int)sizeof(T);
    unpack32(w.x, f + 0 * k, T{});
    unpack32(w.y, f + 1 * k, T{});
    unpack32(w.z, f + 2 * k, T{});
    unpack32(w.w, f + 3 * k, T{});
}

// One row out[j] = src[j] (+ pos[j]) by one warp, scalar (any alignment):
// each lane loads kBatch elements of both rows before it stores any, so the
// loads are not serialised behind stores that may alias them.
template <typename TS, typename TP, typename TO>
__device__ __forceinline__ void scalar_row(const TS* src, int ts, const TP* pos, int tp, bool ok,
                                           TO* out, int H, int lane) {
    constexpr int kBatch = 16;
    for (int j0 = 0; j0 < H; j0 += 32 * kBatch) {
        float v[kBatch], q[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int j = j0 + lane + 32 * u;
            v[u] = 0.0f;
            q[u] = 0.0f;
            if (ok && j < H) {
                v[u] = load_any(src, ts, j);
                if (pos) q[u] = load_any(pos, tp, j);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int j = j0 + lane + 32 * u;
            if (j < H) out[j] = from_f<TO>(pos && ok ? v[u] + q[u] : v[u]);
        }
    }
}

// One cond row by one warp on the vector path: out = cond (f32, 16-byte
// aligned) + pos (TT), all of a lane's loads of a pass issued before its
// stores.
template <typename TT, typename TO>
__device__ __forceinline__ void cond_row_vec(const float* src, const TT* pos, bool ok, TO* out,
                                             int nvec, int lane) {
    constexpr int V = Vec<TT>::n;
    for (int c0 = 0; c0 < nvec; c0 += 32 * kPer) {
        float4 cv[kPer][V / 4];
        uint4 pv[kPer];
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int vi = c0 + lane + 32 * j;
            if (ok && vi < nvec) {
#pragma unroll
                for (int h = 0; h < V / 4; ++h)
                    cv[j][h] = reinterpret_cast<const float4*>(src + (int64_t)vi * V)[h];
                if (pos) pv[j] = ld16(pos + (int64_t)vi * V);
            }
        }
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int vi = c0 + lane + 32 * j;
            if (vi >= nvec) continue;
            float f[V], q[V];
#pragma unroll
            for (int e = 0; e < V; ++e) f[e] = 0.0f;
            if (ok) {
#pragma unroll
                for (int h = 0; h < V / 4; ++h) {
                    f[4 * h] = cv[j][h].x;
                    f[4 * h + 1] = cv[j][h].y;
                    f[4 * h + 2] = cv[j][h].z;
                    f[4 * h + 3] = cv[j][h].w;
                }
                if (pos) {
                    widen<TT>(pv[j], q);
#pragma unroll
                    for (int e = 0; e < V; ++e) f[e] += q[e];
                }
            }
            stv<TO, V>(out + (int64_t)vi * V, f);
        }
    }
}

// Vector path: gathered tables and pos of one type TT, H % V == 0, aligned.
template <typename TT, typename TO>
__global__ void __launch_bounds__(kWarps * 32) k_embed_rows(EmbArgs args) {
    constexpr int V = Vec<TT>::n;
    EmbArgs a = args;
    select_item<TO>(a);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpc = (int)(blockDim.x >> 5);  // warps per CTA: kWarps, or 4 for batched sequences
    const int64_t cta0 = (int64_t)blockIdx.x * wpc * a.rows_per_warp;
    if (threadIdx.x < 2 && cta0 < a.n_rows) {
        // this CTA's ids (thread 0: the last segment's; 1: the position ids)
        int64_t cta1 = cta0 + wpc * a.rows_per_warp;
        cta1 = cta1 < a.n_rows ? cta1 : a.n_rows;
        const int32_t* base = nullptr;
        int64_t lo = 0, hi = 0;
        if (threadIdx.x == 0 && cta1 > a.seg1_end) {
            base = a.seg2.ids;
            lo = (cta0 > a.seg1_end ? cta0 : a.seg1_end) - a.seg1_end;
            hi = cta1 - a.seg1_end;
        } else if (threadIdx.x == 1 && a.pos_ids) {
            base = a.pos_ids;
            lo = cta0;
            hi = cta1;
        }
        if (base) {
            // rounded out to 16-byte blocks, each of which holds a byte of the range
            const uintptr_t s = reinterpret_cast<uintptr_t>(base + lo) & ~uintptr_t(15);
            const uintptr_t e = (reinterpret_cast<uintptr_t>(base + hi) + 15) & ~uintptr_t(15);
            prefetch_l2(reinterpret_cast<const void*>(s), (uint32_t)(e - s));
        }
    }
    grid_dep_wait();
    grid_dep_launch();
    const int64_t w0 = cta0 + (int64_t)warp * a.rows_per_warp;
    int64_t w1 = w0 + a.rows_per_warp;
    w1 = w1 < a.n_rows ? w1 : a.n_rows;
    const int nvec = a.H / V;
    const TT* pos = static_cast<const TT*>(a.pos);
    TO* out = static_cast<TO*>(a.out);
    // cond rows (f32 sources, the sequence's first rows) before the gathered ones
    int64_t g0 = w0;
    for (; g0 < w1 && g0 < a.n_cond; ++g0) {
        int64_t id, p;
        int f;
        row_source(a, g0, &id, &p, &f);
        if (f && lane == 0 && a.err) atomicOr(a.err, f);
        cond_row_vec<TT, TO>(cond_of(args) + g0 * a.H, pos ? pos + p * a.H : nullptr, f == 0,
                             out + g0 * a.H, nvec, lane);
    }
    for (int64_t g = g0; g < w1; g += 32) {
        const int cnt = (int)((w1 - g) < 32 ? (w1 - g) : 32);
        int64_t my_id = 0, my_p = 0;
        int my_f = 0;
        if (lane < cnt) {
            row_source(a, g + lane, &my_id, &my_p, &my_f);
            if (my_f && a.err) atomicOr(a.err, my_f);
        }
        for (int k = 0; k < cnt; k += 2) {
            const bool two = k + 1 < cnt;
            const int64_t ra = g + k, rb = ra + 1;
            const int64_t ida = __shfl_sync(0xffffffffu, my_id, k);
            const int64_t pa = __shfl_sync(0xffffffffu, my_p, k);
            const int fa = __shfl_sync(0xffffffffu, my_f, k);
            const int64_t idb = __shfl_sync(0xffffffffu, my_id, k + 1);
            const int64_t pb = __shfl_sync(0xffffffffu, my_p, k + 1);
            const int fb = two ? __shfl_sync(0xffffffffu, my_f, k + 1) : 1;
            const int sa = seg_of(a, ra), sb = two ? seg_of(a, rb) : 2;  // 1 or 2
            const bool va = fa == 0, vb = two && fb == 0;
            const TT* ta = sa == 1 ? static_cast<const TT*>(a.seg1.table) + ida * a.H
                                   : static_cast<const TT*>(a.seg2.table) + ida * a.H;
            const TT* tb = sb == 1 ? static_cast<const TT*>(a.seg1.table) + idb * a.H
                                   : static_cast<const TT*>(a.seg2.table) + idb * a.H;
            const TT* qa = pos ? pos + pa * a.H : nullptr;
            const TT* qb = pos ? pos + pb * a.H : nullptr;
            for (int c0 = 0; c0 < nvec; c0 += 32 * kPer) {
                uint4 xa[kPer], ya[kPer], xb[kPer], yb[kPer];
#pragma unroll
                for (int j = 0; j < kPer; ++j) {
                    const int vi = c0 + lane + 32 * j;
                    if (vi < nvec) {
                        if (va) {
                            xa[j] = ld16(ta + (int64_t)vi * V);
                            if (qa) ya[j] = ld16(qa + (int64_t)vi * V);
                        }
                        if (vb) {
                            xb[j] = ld16(tb + (int64_t)vi * V);
                            if (qb) yb[j] = ld16(qb + (int64_t)vi * V);
                        }
                    }
                }
                if constexpr (std::is_same<TT, TO>::value && sizeof(TT) == 2) {
                    // same 16-bit type in and out: packed adds, rows copied as is
                    // without a position table, zero rows for bad ids
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        const int vi = c0 + lane + 32 * j;
                        if (vi >= nvec) continue;
                        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                        uint4 oa = va ? (qa ? add16x8<TT>(xa[j], ya[j]) : xa[j]) : z;
                        *reinterpret_cast<uint4*>(out + ra * a.H + (int64_t)vi * V) = oa;
                        if (two) {
                            uint4 ob = vb ? (qb ? add16x8<TT>(xb[j], yb[j]) : xb[j]) : z;
                            *reinterpret_cast<uint4*>(out + rb * a.H + (int64_t)vi * V) = ob;
                        }
                    }
                } else {  // other types: widen to f32, add once, round once
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        const int vi = c0 + lane + 32 * j;
                        if (vi >= nvec) continue;
                        float f[V], q[V];
                        if (va) {
                            widen<TT>(xa[j], f);
                            if (qa) {
                                widen<TT>(ya[j], q);
#pragma unroll
                                for (int e = 0; e < V; ++e) f[e] += q[e];
                            }
                            stv<TO, V>(out + ra * a.H + (int64_t)vi * V, f);
                        } else {  // out-of-range id or position: a zero row
#pragma unroll
                            for (int e = 0; e < V; ++e) f[e] = 0.0f;
                            stv<TO, V>(out + ra * a.H + (int64_t)vi * V, f);
                        }
                        if (vb) {
                            widen<TT>(xb[j], f);
                            if (qb) {
                                widen<TT>(yb[j], q);
#pragma unroll
                                for (int e = 0; e < V; ++e) f[e] += q[e];
                            }
                            stv<TO, V>(out + rb * a.H + (int64_t)vi * V, f);
                        } else if (two) {
#pragma unroll
                            for (int e = 0; e < V; ++e) f[e] = 0.0f;
                            stv<TO, V>(out + rb * a.H + (int64_t)vi * V, f);
                        }
                    }
                }
            }
        }
    }
}

// Any type mix / alignment: scalar, one warp per row.
template <typename TO>
__global__ void __launch_bounds__(256) k_embed_scalar(EmbArgs args, int t1, int t2, int pos_t) {
    EmbArgs a = args;
    select_item<TO>(a);
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    TO* out = static_cast<TO*>(a.out);
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < a.n_rows;
         row += nwarps) {
        int64_t id, p;
        int f;
        row_source(a, row, &id, &p, &f);
        if (f && lane == 0 && a.err) atomicOr(a.err, f);
        const int s = seg_of(a, row);
        const void* src = s == 0 ? static_cast<const void*>(cond_of(args) + row * a.H)
                          : s == 1 ? static_cast<const void*>(
                                         static_cast<const char*>(a.seg1.table) +
                                         id * a.H * (int64_t)type_size(t1))
                                   : static_cast<const void*>(
                                         static_cast<const char*>(a.seg2.table) +
                                         id * a.H * (int64_t)type_size(t2));
        const void* prow = a.pos ? static_cast<const char*>(a.pos) + p * a.H * (int64_t)type_size(pos_t)
                                 : nullptr;
        scalar_row<void, void, TO>(src, s == 0 ? CBX_TYPE_F32 : (s == 1 ? t1 : t2), prow, pos_t,
                                   f == 0, out + row * a.H, a.H, lane);
    }
}

// ------------------------------------------------------------------------
// Batched prefill: B utterances of T tokens, all at positions n_past ..
// n_past + T - 1, so out[b][t] = tok[ids[b][t]] + pos[n_past + t].
//
// The rows are walked position-major (row k = t * B + b): the rows a warp
// takes in sequence share one position row, which it loads once into
// registers and adds to every output row of that position it owns.  Each
// output row then costs one table row from L2 instead of two.  A warp owns
// rows_per_warp consecutive k; each lane loads the id of one row of a group
// of 32 (ids[b][t], L2-prefetched before the PDL wait), and the group is
// taken in chunks of up to NR rows of one position, all NR * NP 16-byte
// token-row loads of a lane issued before any add.
struct BatchArgs {
    const void* tok;
    int64_t n_tok;
    const void* pos;
    int64_t n_pos;
    const int32_t* ids;
    int64_t B, T, n_past, n_rows;
    int H;
    void* out;
    int32_t* err;
    int64_t rows_per_warp;
};

// (t, b) of the row d rows after (t, b) in position-major order.
__device__ __forceinline__ void advance_tb(int64_t B, int64_t t, int64_t b, int64_t d,
                                           int64_t* t_out, int64_t* b_out) {
    int64_t bl = b + d, tl = t;
    if (bl >= B) {
        const int64_t q = bl / B;
        tl += q;
        bl -= q * B;
    }
    *t_out = tl;
    *b_out = bl;
}

// NP = 16-byte vectors of a row per lane (H <= 32 NP V).
template <typename TT, typename TO, int NP>
__global__ void __launch_bounds__(kWarps * 32) k_embed_batched(BatchArgs a) {
    constexpr int V = Vec<TT>::n;
    constexpr int NR = 16 / NP;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t w0 = ((int64_t)blockIdx.x * kWarps + warp) * a.rows_per_warp;
    int64_t w1 = w0 + a.rows_per_warp;
    w1 = w1 < a.n_rows ? w1 : a.n_rows;
    // (t, b) of row w0; advanced row by row below
    int64_t t = w0 < a.n_rows ? w0 / a.B : 0;
    int64_t b = w0 - t * a.B;
    if (w0 < w1 && lane < w1 - w0) {  // the first group's ids, before the wait
        int64_t tl, bl;
        advance_tb(a.B, t, b, lane, &tl, &bl);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.ids + bl * a.T + tl));
    }
    grid_dep_wait();
    grid_dep_launch();
    if (w0 >= w1) return;
    const int nvec = a.H / V;
    const TT* tok = static_cast<const TT*>(a.tok);
    const TT* pos = static_cast<const TT*>(a.pos);
    TO* out = static_cast<TO*>(a.out);
    uint4 q[NP];
    int64_t qt = -1;  // position index whose row q holds
    bool qok = false;
    for (int64_t g = w0; g < w1; g += 32) {
        const int cnt = (int)((w1 - g) < 32 ? (w1 - g) : 32);
        int64_t my_id = 0;
        int my_ok = 0;
        if (lane < cnt) {
            int64_t tl, bl;
            advance_tb(a.B, t, b, lane, &tl, &bl);
            my_id = a.ids[bl * a.T + tl];
            my_ok = my_id >= 0 && my_id < a.n_tok;
            if (!my_ok && a.err) atomicOr(a.err, CBX_EFLAG_TOKEN_OOB);
        }
        for (int j = 0; j < cnt;) {
            int m = cnt - j < NR ? cnt - j : NR;  // rows of this chunk, one position
            if ((int64_t)m > a.B - b) m = (int)(a.B - b);
            if (t != qt) {
                qt = t;
                const int64_t p = a.n_past + t;
                qok = p < a.n_pos;
                if (qok) {
#pragma unroll
                    for (int v = 0; v < NP; ++v) {
                        const int vi = lane + 32 * v;
                        if (vi < nvec) q[v] = ld16(pos + p * a.H + (int64_t)vi * V);
                    }
                } else if (lane == 0 && a.err) {
                    atomicOr(a.err, CBX_EFLAG_POS_OOB);
                }
            }
            uint4 x[NR][NP];
            bool okr[NR];
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const int src = j + (r < m ? r : 0);
                const int64_t id = __shfl_sync(0xffffffffu, my_id, src);
                const int rok = __shfl_sync(0xffffffffu, my_ok, src);
                okr[r] = r < m && qok && rok;
                if (okr[r]) {
#pragma unroll
                    for (int v = 0; v < NP; ++v) {
                        const int vi = lane + 32 * v;
                        if (vi < nvec) x[r][v] = ld16(tok + id * a.H + (int64_t)vi * V);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                if (r >= m) break;
                TO* o = out + ((b + r) * a.T + t) * a.H;
#pragma unroll
                for (int v = 0; v < NP; ++v) {
                    const int vi = lane + 32 * v;
                    if (vi >= nvec) continue;
                    if constexpr (std::is_same<TT, TO>::value && sizeof(TT) == 2) {
                        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                        *reinterpret_cast<uint4*>(o + (int64_t)vi * V) =
                            okr[r] ? add16x8<TT>(x[r][v], q[v]) : z;
                    } else {
                        float f[V], e[V];
#pragma unroll
                        for (int k = 0; k < V; ++k) f[k] = 0.0f;
                        if (okr[r]) {
                            widen<TT>(x[r][v], f);
                            widen<TT>(q[v], e);
#pragma unroll
                            for (int k = 0; k < V; ++k) f[k] += e[k];
                        }
                        stv<TO, V>(o + (int64_t)vi * V, f);
                    }
                }
            }
            j += m;
            b += m;
            if (b == a.B) {
                b = 0;
                ++t;
            }
        }
    }
}

// One wave of 8-warp CTAs, the fewest that give every warp the same number
// of consecutive position-major rows.
template <typename TT, typename TO, int NP>
int launch_batched(BatchArgs a, cudaStream_t st, const char* name) {
    auto kern = k_embed_batched<TT, TO, NP>;
    const int64_t max_warps = (int64_t)num_sms() * occupancy(kern, kWarps * 32) * kWarps;
    a.rows_per_warp = (a.n_rows + max_warps - 1) / max_warps;
    const int64_t warps = (a.n_rows + a.rows_per_warp - 1) / a.rows_per_warp;
    const int64_t blocks = (warps + kWarps - 1) / kWarps;
    return launch_status(launch(kern, dim3((unsigned)blocks), dim3(kWarps * 32), 0, st, a), name);
}

template <typename TT, int NP>
int dispatch_batched(const BatchArgs& a, int out_t, cudaStream_t st, const char* name) {
    switch (out_t) {
        case CBX_TYPE_F32: return launch_batched<TT, float, NP>(a, st, name);
        case CBX_TYPE_BF16: return launch_batched<TT, __nv_bfloat16, NP>(a, st, name);
        default: return launch_batched<TT, __half, NP>(a, st, name);
    }
}

// One wave of CTAs over all n_batch sequences (grid y = sequence); every
// warp owns rows_per_warp consecutive rows of its sequence.  One sequence:
// 8-warp CTAs.  Several: 4-warp CTAs (twice as many resident CTAs, so the
// sequences' CTAs fill the SMs more evenly), and the rows per warp are
// raised until every sequence's CTAs fit in the wave together (when there
// are fewer sequences than resident CTAs).
template <typename TT, typename TO>
int launch_rows(EmbArgs a, int64_t n_batch, cudaStream_t st, const char* name) {
    auto kern = k_embed_rows<TT, TO>;
    const int wpc = n_batch > 1 ? 4 : kWarps;
    const int sms = num_sms();
    const int occ = occupancy(kern, wpc * 32);
    const int64_t max_ctas = (int64_t)sms * occ;
    const int64_t max_warps = max_ctas * wpc;
    int64_t rpw = (a.n_rows * n_batch + max_warps - 1) / max_warps;
    if (n_batch > 1) {
        const int64_t per_seq = max_ctas / n_batch;  // CTAs per sequence in one wave
        const int64_t need = per_seq > 0 ? (a.n_rows + wpc * per_seq - 1) / (wpc * per_seq)
                                         : (a.n_rows + wpc - 1) / wpc;
        if (rpw < need) rpw = need;
    }
    a.rows_per_warp = rpw;
    const int64_t rows_per_cta = rpw * wpc;
    const int64_t blocks = (a.n_rows + rows_per_cta - 1) / rows_per_cta;
    return launch_status(
        launch(kern, dim3((unsigned)blocks, (unsigned)n_batch), dim3(wpc * 32), 0, st, a), name);
}

template <typename TT>
int dispatch_vec(const EmbArgs& a, int64_t n_batch, int out_t, cudaStream_t st, const char* name) {
    switch (out_t) {
        case CBX_TYPE_F32: return launch_rows<TT, float>(a, n_batch, st, name);
        case CBX_TYPE_BF16: return launch_rows<TT, __nv_bfloat16>(a, n_batch, st, name);
        default: return launch_rows<TT, __half>(a, n_batch, st, name);
    }
}

int launch_scalar(const EmbArgs& a, int64_t n_batch, int out_t, int t1, int t2, int pos_t,
                  cudaStream_t st, const char* name) {
    const int sms = num_sms();
    int64_t blocks = (a.n_rows + 7) / 8;
    int64_t cap = (int64_t)sms * 8 / n_batch;
    if (cap < 1) cap = 1;
    if (blocks > cap) blocks = cap;
    const dim3 grid((unsigned)blocks, (unsigned)n_batch);
    cudaError_t e;
    switch (out_t) {
        case CBX_TYPE_F32:
            e = launch(k_embed_scalar<float>, grid, dim3(256), 0, st, a, t1, t2, pos_t);
            break;
        case CBX_TYPE_BF16:
            e = launch(k_embed_scalar<__nv_bfloat16>, grid, dim3(256), 0, st, a, t1, t2, pos_t);
            break;
        default:
            e = launch(k_embed_scalar<__half>, grid, dim3(256), 0, st, a, t1, t2, pos_t);
    }
    return launch_status(e, name);
}

// Picks the vector kernel when every gathered table and pos share one type,
// H is a whole number of 16-byte vectors and the tables and output are
// 16-byte aligned; else the scalar kernel.  t1 < 0: no seg1.  n_batch
// sequences of a.n_rows rows each (grid y; at most 65535).
int run(const EmbArgs& a, int t1, int t2, int pos_t, int out_t, cudaStream_t st,
        const char* name, int64_t n_batch = 1) {
    const int V = t2 == CBX_TYPE_F32 ? 4 : 8;
    const int osz = type_size(out_t);
    const bool vec = (t1 < 0 || t1 == t2) && (!a.pos || pos_t == t2) && a.H % V == 0 &&
                     (a.n_cond == 0 || aligned16(a.cond)) &&
                     aligned16(a.seg2.table) && (t1 < 0 || aligned16(a.seg1.table)) &&
                     (!a.pos || aligned16(a.pos)) && aligned16(a.out) &&
                     ((int64_t)a.H * osz) % 16 == 0 && (V * osz) >= 8;
    if (!vec) return launch_scalar(a, n_batch, out_t, t1 < 0 ? t2 : t1, t2, pos_t, st, name);
    switch (t2) {
        case CBX_TYPE_F32: return dispatch_vec<float>(a, n_batch, out_t, st, name);
        case CBX_TYPE_BF16: return dispatch_vec<__nv_bfloat16>(a, n_batch, out_t, st, name);
        default: return dispatch_vec<__half>(a, n_batch, out_t, st, name);
    }
}

// Batched prefill: the position-major kernel when the token and position
// tables share one type, rows are whole 16-byte vectors (at most 256 per
// row), and tables and output are 16-byte aligned; else the row kernels
// with the position of output row r = b T + t taken as n_past + r % T.
int run_batched(const BatchArgs& b, int tok_t, int pos_t, int out_t, cudaStream_t st,
                const char* name) {
    const int V = tok_t == CBX_TYPE_F32 ? 4 : 8;
    const int osz = type_size(out_t);
    const int64_t nvec = b.H / V;
    const bool vec = b.pos && pos_t == tok_t && b.H % V == 0 && nvec <= 256 &&
                     aligned16(b.tok) && aligned16(b.pos) && aligned16(b.out) &&
                     ((int64_t)b.H * osz) % 16 == 0 && (V * osz) >= 8;
    if (vec) {
        const bool np4 = nvec <= 128;
        switch (tok_t) {
            case CBX_TYPE_F32:
                return np4 ? dispatch_batched<float, 4>(b, out_t, st, name)
                           : dispatch_batched<float, 8>(b, out_t, st, name);
            case CBX_TYPE_BF16:
                return np4 ? dispatch_batched<__nv_bfloat16, 4>(b, out_t, st, name)
                           : dispatch_batched<__nv_bfloat16, 8>(b, out_t, st, name);
            default:
                return np4 ? dispatch_batched<__half, 4>(b, out_t, st, name)
                           : dispatch_batched<__half, 8>(b, out_t, st, name);
        }
    }
    EmbArgs a{};
    a.seg2 = Seg{b.tok, b.n_tok, b.ids};
    a.pos = b.pos;
    a.n_pos = b.n_pos;
    a.pos_offset = b.n_past;
    a.pos_period = b.T;
    a.n_rows = b.n_rows;
    a.H = b.H;
    a.out = b.out;
    a.err = b.err;
    return run(a, -1, tok_t, pos_t, out_t, st, name);
}

}  // namespace
}  // namespace cbx

extern "C" CBX_API int cbx_embed_gather_add(const void* tok_table, int tok_type, int64_t n_tok_rows,
                                            const void* pos_table, int pos_type,
                                            int64_t n_pos_rows, const int32_t* ids,
                                            const int32_t* pos_ids, int64_t pos_offset,
                                            int64_t n_rows, int64_t hidden, void* out,
                                            int out_type, int32_t* err_word,
                                            cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_embed_gather_add";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n_rows < 0 || hidden <= 0 || n_tok_rows < 0 || n_pos_rows < 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_rows %lld hidden %lld", name, (long long)n_rows,
                    (long long)hidden);
    if (hidden > INT32_MAX) return fail(CBX_ERR_INVALID_ARG, "%s: hidden too large", name);
    if (!valid_type(tok_type) || !valid_type(out_type) || (pos_table && !valid_type(pos_type)))
        return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: types tok %d pos %d out %d", name, tok_type,
                    pos_type, out_type);
    if (n_rows == 0) return ok();
    if (!tok_table || !ids || !out) return fail(CBX_ERR_INVALID_ARG, "%s: NULL pointer", name);
    EmbArgs a{};
    a.seg2 = Seg{tok_table, n_tok_rows, ids};
    a.pos = pos_table;
    a.n_pos = n_pos_rows;
    a.pos_ids = pos_ids;
    a.pos_offset = pos_offset;
    a.n_rows = n_rows;
    a.H = (int)hidden;
    a.out = out;
    a.err = err_word;
    return run(a, -1, tok_type, pos_type, out_type, st, name);
}

namespace cbx {
namespace {

// The prefill sequence for n_batch utterances laid out back to back (cond
// rows [n_batch][n_cond][hidden], ids [n_batch][n], out [n_batch][N][hidden]);
// n_batch = 1 is cbx_t3_embed_sequence.
int embed_sequences(const float* cond_rows, int64_t n_cond, const void* prompt_table,
                    int prompt_type, int64_t n_prompt_table_rows, const int32_t* prompt_ids,
                    int64_t n_prompt, const void* tok_table, int tok_type, int64_t n_tok_table_rows,
                    const int32_t* tok_ids, int64_t n_tok, const void* pos_table, int pos_type,
                    int64_t n_pos_rows, int64_t n_past, int64_t hidden, int64_t n_batch, void* out,
                    int out_type, int32_t* err_word, cudaStream_t st, const char* name) {
    if (n_cond < 0 || n_prompt < 0 || n_tok < 0 || hidden <= 0 || n_prompt_table_rows < 0 ||
        n_tok_table_rows < 0 || n_pos_rows < 0 || n_past < 0 || n_batch < 0)
        return fail(CBX_ERR_INVALID_ARG,
                    "%s: n_cond %lld n_prompt %lld n_tok %lld hidden %lld n_past %lld n_batch %lld",
                    name, (long long)n_cond, (long long)n_prompt, (long long)n_tok,
                    (long long)hidden, (long long)n_past, (long long)n_batch);
    if (hidden > INT32_MAX) return fail(CBX_ERR_INVALID_ARG, "%s: hidden too large", name);
    if (!valid_type(out_type) || (n_tok && !valid_type(tok_type)) ||
        (n_prompt && !valid_type(prompt_type)) || (pos_table && !valid_type(pos_type)))
        return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: types prompt %d tok %d pos %d out %d", name,
                    prompt_type, tok_type, pos_type, out_type);
    const int64_t n_rows = n_cond + n_prompt + n_tok;
    if (n_rows == 0 || n_batch == 0) return ok();
    if (n_batch > INT64_MAX / n_rows / hidden)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_batch * rows * hidden overflows", name);
    if (!out || (n_cond && !cond_rows) || (n_prompt && (!prompt_table || !prompt_ids)) ||
        (n_tok && (!tok_table || !tok_ids)))
        return fail(CBX_ERR_INVALID_ARG, "%s: NULL pointer", name);
    EmbArgs a{};
    a.cond = cond_rows;
    a.n_cond = n_cond;
    a.seg1 = Seg{prompt_table, n_prompt_table_rows, prompt_ids};
    a.seg1_end = n_cond + n_prompt;
    // with no text tokens the prompt segment carries the vector path's type
    a.seg2 = n_tok ? Seg{tok_table, n_tok_table_rows, tok_ids}
                   : Seg{prompt_table, n_prompt_table_rows, prompt_ids};
    a.pos = pos_table;
    a.n_pos = n_pos_rows;
    a.pos_offset = n_past;
    a.n_rows = n_rows;
    a.H = (int)hidden;
    a.out = out;
    a.err = err_word;
    a.cond_bstride = n_cond * hidden;
    a.seg1_bstride = n_prompt;
    a.seg2_bstride = n_tok ? n_tok : n_prompt;
    a.out_bstride = n_rows * hidden;
    const int t2 = n_tok ? tok_type : (n_prompt ? prompt_type : (pos_table ? pos_type : CBX_TYPE_F32));
    const int t1 = n_prompt ? prompt_type : -1;
    if (!a.seg2.table) a.seg2.table = out;  // cond rows only: any aligned pointer (never read)
    // at most 65535 utterances per launch (grid y)
    constexpr int64_t kMaxY = 65535;
    const int64_t osz = type_size(out_type);
    for (int64_t c0 = 0; c0 < n_batch; c0 += kMaxY) {
        const int64_t nb = n_batch - c0 < kMaxY ? n_batch - c0 : kMaxY;
        EmbArgs c = a;
        if (c0) {
            if (c.cond) c.cond += c0 * a.cond_bstride;
            if (c.seg1.ids) c.seg1.ids += c0 * a.seg1_bstride;
            if (c.seg2.ids) c.seg2.ids += c0 * a.seg2_bstride;
            c.out = static_cast<char*>(out) + c0 * a.out_bstride * osz;
        }
        const int rc = run(c, t1, t2, pos_table ? pos_type : t2, out_type, st, name, nb);
        if (rc != CBX_OK) return rc;
    }
    return ok();
}

}  // namespace
}  // namespace cbx

extern "C" CBX_API int cbx_t3_embed_sequence(const float* cond_rows, int64_t n_cond,
                                             const void* prompt_table, int prompt_type,
                                             int64_t n_prompt_table_rows,
                                             const int32_t* prompt_ids, int64_t n_prompt,
                                             const void* tok_table, int tok_type,
                                             int64_t n_tok_table_rows, const int32_t* tok_ids,
                                             int64_t n_tok, const void* pos_table, int pos_type,
                                             int64_t n_pos_rows, int64_t n_past, int64_t hidden,
                                             void* out, int out_type, int32_t* err_word,
                                             cbx_stream_t stream) {
    return cbx::embed_sequences(cond_rows, n_cond, prompt_table, prompt_type, n_prompt_table_rows,
                                prompt_ids, n_prompt, tok_table, tok_type, n_tok_table_rows,
                                tok_ids, n_tok, pos_table, pos_type, n_pos_rows, n_past, hidden, 1,
                                out, out_type, err_word, reinterpret_cast<cudaStream_t>(stream),
                                "cbx_t3_embed_sequence");
}

extern "C" CBX_API int cbx_t3_embed_sequence_batched(
    const float* cond_rows, int64_t n_cond, const void* prompt_table, int prompt_type,
    int64_t n_prompt_table_rows, const int32_t* prompt_ids, int64_t n_prompt, const void* tok_table,
    int tok_type, int64_t n_tok_table_rows, const int32_t* tok_ids, int64_t n_tok,
    const void* pos_table, int pos_type, int64_t n_pos_rows, int64_t n_past, int64_t hidden,
    int64_t n_batch, void* out, int out_type, int32_t* err_word, cbx_stream_t stream) {
    return cbx::embed_sequences(cond_rows, n_cond, prompt_table, prompt_type, n_prompt_table_rows,
                                prompt_ids, n_prompt, tok_table, tok_type, n_tok_table_rows,
                                tok_ids, n_tok, pos_table, pos_type, n_pos_rows, n_past, hidden,
                                n_batch, out, out_type, err_word,
                                reinterpret_cast<cudaStream_t>(stream),
                                "cbx_t3_embed_sequence_batched");
}

extern "C" CBX_API int cbx_embed_gather_add_batched(const void* tok_table, int tok_type,
                                                    int64_t n_tok_rows, const void* pos_table,
                                                    int pos_type, int64_t n_pos_rows,
                                                    const int32_t* ids, int64_t n_batch,
                                                    int64_t seq_len, int64_t n_past,
                                                    int64_t hidden, void* out, int out_type,
                                                    int32_t* err_word, cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_embed_gather_add_batched";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n_batch < 0 || seq_len < 0 || n_past < 0 || hidden <= 0 || n_tok_rows < 0 ||
        n_pos_rows < 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_batch %lld seq_len %lld n_past %lld hidden %lld",
                    name, (long long)n_batch, (long long)seq_len, (long long)n_past,
                    (long long)hidden);
    if (hidden > INT32_MAX) return fail(CBX_ERR_INVALID_ARG, "%s: hidden too large", name);
    if (seq_len > 0 && n_batch > INT64_MAX / seq_len / hidden)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_batch * seq_len * hidden overflows", name);
    if (!valid_type(tok_type) || !valid_type(out_type) || (pos_table && !valid_type(pos_type)))
        return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: types tok %d pos %d out %d", name, tok_type,
                    pos_type, out_type);
    const int64_t n_rows = n_batch * seq_len;
    if (n_rows == 0) return ok();
    if (!tok_table || !ids || !out) return fail(CBX_ERR_INVALID_ARG, "%s: NULL pointer", name);
    BatchArgs b{};
    b.tok = tok_table;
    b.n_tok = n_tok_rows;
    b.pos = pos_table;
    b.n_pos = n_pos_rows;
    b.ids = ids;
    b.B = n_batch;
    b.T = seq_len;
    b.n_past = n_past;
    b.n_rows = n_rows;
    b.H = (int)hidden;
    b.out = out;
    b.err = err_word;
    return run_batched(b, tok_type, pos_type, out_type, st, name);
}
