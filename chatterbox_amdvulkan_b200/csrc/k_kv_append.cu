// k_kv_append.cu — the T3 attention prologue after the QKV GEMM, fused:
// qkv bias add, the Q copy, and the K / V writes into the KV cache.
//
// The engine (chatterbox-cpp/src/t3.cpp:465-489) emits
//   cur = ggml_add(mul_mat(qkv_w, x), qkv_b)            f32, rounded once
//   Qcur / Kcur / Vcur = views of rows [0, D), [D, 2D), [2D, 3D) of cur
//   ggml_cpy(Kcur -> cache_k[il][n_past + i]),  ggml_cpy(Vcur -> cache_v[...])
//   Q = ggml_cont(Qcur)
// i.e. four memory passes; here it is one: read the GEMM output row (3D f32)
// and the bias, write Q (D f32) and the K and V rows of the cache, converted
// to the cache's element type (the engine's cache is f32, t3.cpp:252-253; f16
// and bf16 caches halve the attention's cache reads).  Bit-exact: one f32 add,
// one rounding to the cache type.
//
// Rows are independent tokens: a prefill chunk of one stream (positions
// n_past + i, one cache slab) or one new token per stream of a batched decode
// step (positions[r], slab r).  A row whose position is outside
// [0, max_context) writes no cache row and raises CBX_EFLAG_POS_OOB in the
// caller's error word; its Q row is still written.
#include "cbx_common.cuh"

namespace cbx {
namespace {

constexpr int kThreads = 256;

struct KvArgs {
    const float* qkv;
    int64_t qkv_stride;
    const float* bias;
    int64_t n_rows;
    int D;
    const int32_t* positions;
    int32_t pos_offset;
    void* ck;
    void* cv;
    int64_t slab_stride;
    int64_t max_context;
    float* q;
    int32_t* err;
};

// D % 4 == 0, qkv / bias / q 16-byte aligned, caches 8- (16-bit) or
// 16-byte (f32) aligned: one float4 of each of Q, K, V per thread and step.
// Grid (chunks of a row, rows).
template <typename TC>
__global__ void __launch_bounds__(kThreads) k_qkv_kv_append_vec(KvArgs a) {
    const int nv = a.D / 4;
    const int vi = blockIdx.x * kThreads + threadIdx.x;
    if (threadIdx.x == 0 && blockIdx.y < a.n_rows) {
        const int n = nv - blockIdx.x * kThreads < kThreads ? nv - blockIdx.x * kThreads : kThreads;
        if (n > 0) {
            const float* row = a.qkv + (int64_t)blockIdx.y * a.qkv_stride + blockIdx.x * kThreads * 4;
            prefetch_l2(row, (uint32_t)n * 16u);
            prefetch_l2(row + a.D, (uint32_t)n * 16u);
            prefetch_l2(row + 2 * a.D, (uint32_t)n * 16u);
        }
    }
    grid_dep_wait();
    grid_dep_launch();
    if (vi >= nv) return;
    float bq[4] = {0.f, 0.f, 0.f, 0.f}, bk[4] = {0.f, 0.f, 0.f, 0.f}, bv[4] = {0.f, 0.f, 0.f, 0.f};
    if (a.bias) {
        ldv<float, 4>(a.bias + vi * 4, bq);
        ldv<float, 4>(a.bias + a.D + vi * 4, bk);
        ldv<float, 4>(a.bias + 2 * a.D + vi * 4, bv);
    }
    for (int64_t r = blockIdx.y; r < a.n_rows; r += gridDim.y) {
        const float* row = a.qkv + r * a.qkv_stride;
        float q[4], k[4], v[4];
        ldv<float, 4>(row + vi * 4, q);
        ldv<float, 4>(row + a.D + vi * 4, k);
        ldv<float, 4>(row + 2 * a.D + vi * 4, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            q[j] = __fadd_rn(q[j], bq[j]);
            k[j] = __fadd_rn(k[j], bk[j]);
            v[j] = __fadd_rn(v[j], bv[j]);
        }
        if (a.q) stv<float, 4>(a.q + r * a.D + vi * 4, q);
        const int64_t pos = a.positions ? (int64_t)__ldg(a.positions + r) : a.pos_offset + r;
        if (pos < 0 || pos >= a.max_context) {
            if (vi == 0) atomicOr(a.err, CBX_EFLAG_POS_OOB);
            continue;
        }
        const int64_t off = r * a.slab_stride + pos * a.D + vi * 4;
        stv<TC, 4>(static_cast<TC*>(a.ck) + off, k);
        stv<TC, 4>(static_cast<TC*>(a.cv) + off, v);
    }
}

// Any D / alignment: one element of each of Q, K, V per thread.
template <typename TC>
__global__ void __launch_bounds__(kThreads) k_qkv_kv_append_scalar(KvArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * kThreads + threadIdx.x;
    if (i >= a.D) return;
    const float bq = a.bias ? __ldg(a.bias + i) : 0.0f;
    const float bk = a.bias ? __ldg(a.bias + a.D + i) : 0.0f;
    const float bv = a.bias ? __ldg(a.bias + 2 * a.D + i) : 0.0f;
    for (int64_t r = blockIdx.y; r < a.n_rows; r += gridDim.y) {
        const float* row = a.qkv + r * a.qkv_stride;
        const float q = __fadd_rn(__ldg(row + i), bq);
        const float k = __fadd_rn(__ldg(row + a.D + i), bk);
        const float v = __fadd_rn(__ldg(row + 2 * a.D + i), bv);
        if (a.q) a.q[r * a.D + i] = q;
        const int64_t pos = a.positions ? (int64_t)__ldg(a.positions + r) : a.pos_offset + r;
        if (pos < 0 || pos >= a.max_context) {
            if (i == 0) atomicOr(a.err, CBX_EFLAG_POS_OOB);
            continue;
        }
        const int64_t off = r * a.slab_stride + pos * a.D + i;
        static_cast<TC*>(a.ck)[off] = from_f<TC>(k);
        static_cast<TC*>(a.cv)[off] = from_f<TC>(v);
    }
}

template <typename TC>
int run_kv(const KvArgs& a, cudaStream_t st) {
    const int cache_align = sizeof(TC) == 4 ? 16 : 8;
    const bool vec = a.D % 4 == 0 && a.qkv_stride % 4 == 0 && aligned16(a.qkv) &&
                     (!a.bias || aligned16(a.bias)) && (!a.q || aligned16(a.q)) &&
                     (reinterpret_cast<uintptr_t>(a.ck) % cache_align) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.cv) % cache_align) == 0 &&
                     (a.slab_stride * (int64_t)sizeof(TC)) % cache_align == 0;
    const int per_cta = vec ? kThreads * 4 : kThreads;
    const unsigned gx = (unsigned)((a.D + per_cta - 1) / per_cta);
    const unsigned gy = (unsigned)(a.n_rows < 65535 ? a.n_rows : 65535);
    cudaError_t e = vec ? launch(k_qkv_kv_append_vec<TC>, dim3(gx, gy), dim3(kThreads), 0, st, a)
                        : launch(k_qkv_kv_append_scalar<TC>, dim3(gx, gy), dim3(kThreads), 0, st, a);
    return launch_status(e, "cbx_qkv_kv_append");
}

}  // namespace
}  // namespace cbx

// t3.cpp:465-489: qkv bias add, Q copy, K / V cache writes.
extern "C" CBX_API int cbx_qkv_kv_append(const float* qkv, int64_t qkv_row_stride,
                                         const float* qkv_bias, int64_t n_rows, int64_t D,
                                         const int32_t* positions, int32_t pos_offset,
                                         void* cache_k, void* cache_v, int cache_type,
                                         int64_t slab_stride, int64_t max_context, float* q_out,
                                         int32_t* err_word, cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_qkv_kv_append";
    if (n_rows < 0 || D <= 0 || D > (1 << 24))
        return fail(CBX_ERR_INVALID_ARG, "%s: n_rows %lld D %lld", name, (long long)n_rows,
                    (long long)D);
    if (qkv_row_stride == 0) qkv_row_stride = 3 * D;
    if (qkv_row_stride < 3 * D)
        return fail(CBX_ERR_INVALID_ARG, "%s: qkv_row_stride %lld < 3 D", name,
                    (long long)qkv_row_stride);
    if (max_context <= 0 || slab_stride < 0)
        return fail(CBX_ERR_INVALID_ARG, "%s: max_context %lld slab_stride %lld", name,
                    (long long)max_context, (long long)slab_stride);
    if (n_rows > 1 && slab_stride != 0 && slab_stride < max_context * D)
        return fail(CBX_ERR_INVALID_ARG,
                    "%s: slab_stride %lld < max_context * D = %lld: the rows' slabs overlap", name,
                    (long long)slab_stride, (long long)(max_context * D));
    if (!valid_type(cache_type))
        return fail(CBX_ERR_UNSUPPORTED_DTYPE, "%s: cache_type %d", name, cache_type);
    if (n_rows == 0) return ok();
    if (!qkv || !cache_k || !cache_v || !err_word)
        return fail(CBX_ERR_INVALID_ARG, "%s: NULL qkv, cache or err_word", name);
    KvArgs a{qkv, qkv_row_stride, qkv_bias, n_rows, (int)D, positions, pos_offset, cache_k,
             cache_v, slab_stride, max_context, q_out, err_word};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    switch (cache_type) {
        case CBX_TYPE_F32: return run_kv<float>(a, st);
        case CBX_TYPE_BF16: return run_kv<__nv_bfloat16>(a, st);
        default: return run_kv<__half>(a, st);
    }
}
