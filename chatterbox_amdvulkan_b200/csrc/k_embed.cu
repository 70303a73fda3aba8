// k_embed.cu — token + learned-position embedding gather-add.
//
// One warp per output row: the row's token id and position are broadcast
// loads, the two table rows are read with 16-byte vector loads (the tables —
// 6563 x 1024 speech tokens, 4096 x 1024 positions — stay L2-resident across
// rows), widened to f32, added once, rounded once to the output type and
// written with vector stores.  Compulsory HBM traffic is the output, the ids
// and each distinct table row once.
#include <type_traits>

#include "cbx_common.cuh"

namespace cbx {
namespace {

struct EmbArgs {
    const void* tok;
    int64_t n_tok;
    const void* pos;
    int64_t n_pos;
    const int32_t* ids;
    const int32_t* pos_ids;
    int64_t pos_offset;
    int64_t n_rows;
    int H;
    void* out;
    int32_t* err;
};

// Vector path: tok and pos of the same type TT, H % V == 0, aligned.
template <typename TT, typename TO>
__global__ void __launch_bounds__(256) k_embed_vec(EmbArgs a) {
    constexpr int V = Vec<TT>::n;
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int nvec = a.H / V;
    const TT* tok = static_cast<const TT*>(a.tok);
    const TT* pos = static_cast<const TT*>(a.pos);
    TO* out = static_cast<TO*>(a.out);
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < a.n_rows;
         row += nwarps) {
        const int64_t id = a.ids[row];
        const int64_t p = a.pos_ids ? (int64_t)a.pos_ids[row] : a.pos_offset + row;
        const bool bad_t = id < 0 || id >= a.n_tok;
        const bool bad_p = pos && (p < 0 || p >= a.n_pos);
        TO* orow = out + row * a.H;
        if (bad_t || bad_p) {
            if (lane == 0 && a.err)
                atomicOr(a.err, (bad_t ? CBX_EFLAG_TOKEN_OOB : 0) | (bad_p ? CBX_EFLAG_POS_OOB : 0));
            float z[V];
#pragma unroll
            for (int j = 0; j < V; ++j) z[j] = 0.0f;
            for (int vi = lane; vi < nvec; vi += 32) stv<TO, V>(orow + (int64_t)vi * V, z);
            continue;
        }
        const TT* trow = tok + id * a.H;
        const TT* prow = pos ? pos + p * a.H : nullptr;
        for (int vi = lane; vi < nvec; vi += 64) {
            // two vectors per lane per iteration: four loads in flight
            float t0[V], t1[V], q0[V], q1[V];
            const int vj = vi + 32;
            const bool two = vj < nvec;
            ldv<TT, V>(trow + (int64_t)vi * V, t0);
            if (two) ldv<TT, V>(trow + (int64_t)vj * V, t1);
            if (prow) {
                ldv<TT, V>(prow + (int64_t)vi * V, q0);
                if (two) ldv<TT, V>(prow + (int64_t)vj * V, q1);
#pragma unroll
                for (int j = 0; j < V; ++j) t0[j] += q0[j];
                if (two) {
#pragma unroll
                    for (int j = 0; j < V; ++j) t1[j] += q1[j];
                }
            }
            stv<TO, V>(orow + (int64_t)vi * V, t0);
            if (two) stv<TO, V>(orow + (int64_t)vj * V, t1);
        }
    }
}

__device__ __forceinline__ float load_any(const void* p, int type, int64_t i) {
    if (type == CBX_TYPE_F32) return static_cast<const float*>(p)[i];
    if (type == CBX_TYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// Any type mix / alignment: scalar, one warp per row.
template <typename TO>
__global__ void __launch_bounds__(256) k_embed_scalar(EmbArgs a, int tok_t, int pos_t) {
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    TO* out = static_cast<TO*>(a.out);
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < a.n_rows;
         row += nwarps) {
        const int64_t id = a.ids[row];
        const int64_t p = a.pos_ids ? (int64_t)a.pos_ids[row] : a.pos_offset + row;
        const bool bad_t = id < 0 || id >= a.n_tok;
        const bool bad_p = a.pos && (p < 0 || p >= a.n_pos);
        if ((bad_t || bad_p) && lane == 0 && a.err)
            atomicOr(a.err, (bad_t ? CBX_EFLAG_TOKEN_OOB : 0) | (bad_p ? CBX_EFLAG_POS_OOB : 0));
        TO* orow = out + row * a.H;
        for (int j = lane; j < a.H; j += 32) {
            float v = 0.0f;
            if (!bad_t && !bad_p) {
                v = load_any(a.tok, tok_t, id * a.H + j);
                if (a.pos) v += load_any(a.pos, pos_t, p * a.H + j);
            }
            orow[j] = from_f<TO>(v);
        }
    }
}

template <typename K>
int launch_rows(K kern, const EmbArgs& a, cudaStream_t st, int extra0 = -1, int extra1 = -1) {
    const int sms = num_sms();
    int wpc;
    if (a.n_rows >= (int64_t)sms * 16) wpc = 8;
    else if (a.n_rows >= (int64_t)sms * 4) wpc = 4;
    else if (a.n_rows >= (int64_t)sms * 2) wpc = 2;
    else wpc = 1;
    const int threads = wpc * 32;
    const int occ = occupancy(kern, threads);
    int64_t blocks = (a.n_rows + wpc - 1) / wpc;
    const int64_t cap = (int64_t)sms * occ;
    if (blocks > cap) blocks = cap;
    cudaError_t e;
    if constexpr (std::is_same<K, void (*)(EmbArgs)>::value)
        e = launch(kern, dim3((unsigned)blocks), dim3(threads), 0, st, a);
    else
        e = launch(kern, dim3((unsigned)blocks), dim3(threads), 0, st, a, extra0, extra1);
    return launch_status(e, "cbx_embed_gather_add");
}

template <typename TT>
int dispatch_vec(const EmbArgs& a, int out_t, cudaStream_t st) {
    switch (out_t) {
        case CBX_TYPE_F32: return launch_rows(k_embed_vec<TT, float>, a, st);
        case CBX_TYPE_BF16: return launch_rows(k_embed_vec<TT, __nv_bfloat16>, a, st);
        default: return launch_rows(k_embed_vec<TT, __half>, a, st);
    }
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
    EmbArgs a{tok_table, n_tok_rows, pos_table, n_pos_rows, ids, pos_ids, pos_offset,
              n_rows,    (int)hidden, out,      err_word};
    const int V = tok_type == CBX_TYPE_F32 ? 4 : 8;
    const int osz = type_size(out_type);
    const bool vec = (!pos_table || pos_type == tok_type) && hidden % V == 0 &&
                     aligned16(tok_table) && (!pos_table || aligned16(pos_table)) &&
                     aligned16(out) && (hidden * osz) % 16 == 0 && (V * osz) >= 8;
    if (vec) {
        switch (tok_type) {
            case CBX_TYPE_F32: return dispatch_vec<float>(a, out_type, st);
            case CBX_TYPE_BF16: return dispatch_vec<__nv_bfloat16>(a, out_type, st);
            default: return dispatch_vec<__half>(a, out_type, st);
        }
    }
    switch (out_type) {
        case CBX_TYPE_F32: return launch_rows(k_embed_scalar<float>, a, st, tok_type, pos_type);
        case CBX_TYPE_BF16:
            return launch_rows(k_embed_scalar<__nv_bfloat16>, a, st, tok_type, pos_type);
        default: return launch_rows(k_embed_scalar<__half>, a, st, tok_type, pos_type);
    }
}
