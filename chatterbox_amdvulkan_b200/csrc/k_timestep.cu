// k_timestep.cu — batched sinusoidal timestep embedding (+ SiLU).
//
// The engine computes this on the host for one scalar t per call
// (chatterbox-cpp/src/cfm_decoder.cpp:49-62); here a batch of n_t values is
// embedded in one launch, one thread per output element.  The argument
// a = (scale * t) * freq is formed in f32 in the engine's order so that the
// phase of sin/cos at |a| ~ 1000 rad matches the host expression; freq is the
// table of cbx_sinusoid_freqs (the engine's f32 host expression).
#include "cbx_common.cuh"

namespace cbx {
namespace {

template <bool SILU>
__global__ void __launch_bounds__(256) k_timestep(const float* t, int64_t n_t, const float* freqs,
                                                  int dim, float scale, float* y) {
    grid_dep_wait();
    grid_dep_launch();
    const int half = dim >> 1;
    const int64_t n = n_t * dim;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / dim;
        const int j = (int)(e - i * dim);
        float v = 0.0f;
        if (j < 2 * half) {
            const int jj = j < half ? j : j - half;
            const float a = __fmul_rn(__fmul_rn(scale, __ldg(t + i)), __ldg(freqs + jj));
            v = j < half ? sinf(a) : cosf(a);
        }
        if (SILU) v = silu_f(v);
        y[e] = v;
    }
}

}  // namespace
}  // namespace cbx

extern "C" CBX_API int cbx_timestep_embed(const float* t, int64_t n_t, const float* freqs,
                                          int32_t dim, float scale, int act, float* y,
                                          cbx_stream_t stream) {
    using namespace cbx;
    const char* name = "cbx_timestep_embed";
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (n_t < 0 || dim < 4)
        return fail(CBX_ERR_INVALID_ARG, "%s: n_t %lld dim %d (dim must be >= 4)", name,
                    (long long)n_t, (int)dim);
    if (act != CBX_ACT_NONE && act != CBX_ACT_SILU)
        return fail(CBX_ERR_INVALID_ARG, "%s: act %d (NONE or SILU)", name, act);
    if (n_t == 0) return ok();
    if (!t || !freqs || !y) return fail(CBX_ERR_INVALID_ARG, "%s: NULL pointer", name);
    const int64_t n = n_t * dim;
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    cudaError_t e = act == CBX_ACT_SILU
                        ? launch(k_timestep<true>, dim3((unsigned)blocks), dim3(256), 0, st, t,
                                 n_t, freqs, (int)dim, scale, y)
                        : launch(k_timestep<false>, dim3((unsigned)blocks), dim3(256), 0, st, t,
                                 n_t, freqs, (int)dim, scale, y);
    return launch_status(e, name);
}
