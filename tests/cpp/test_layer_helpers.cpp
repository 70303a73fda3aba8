// GPU test of the C++ helper mirror (include/cbx_layer_helpers.hpp) against the
// CPU oracle (oracle/libcbx_oracle.so, test infrastructure).  Built and run by
// tests/test_cpp_helpers.py; exits 0 when every check passes.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "cbx_layer_helpers.hpp"

extern "C" {  // oracle/cbx_oracle.c
int cbxo_add_layernorm_act(const void*, const void*, int, int64_t, const float*, const float*, float,
                           int64_t, int64_t, void*, void*, int, int64_t, int, const float*);
int cbxo_layernorm_channels(const float*, const float*, const float*, float, const float*, int64_t,
                            int64_t, int64_t, int, int, float*);
int cbxo_snake(const float*, const float*, const float*, float, int64_t, int64_t, int64_t, int,
               float*);
int cbxo_gelu_tanh(const void*, void*, int64_t, int);
int cbxo_mish(const void*, void*, int64_t, int);
int cbxo_embed_gather_add(const void*, int, int64_t, const void*, int, int64_t, const int32_t*,
                          const int32_t*, int64_t, int64_t, int64_t, void*, int, int32_t*);
int cbxo_sinusoid_freqs(int32_t, float*);
int cbxo_gelu_erf(const void*, void*, int64_t, int);
int cbxo_bias_act(const void*, void*, int, int64_t, int64_t, const float*, int, int64_t, int, float);
int cbxo_sum3_scale(const void*, const void*, const void*, float, void*, int64_t, int);
int cbxo_qkv_kv_append(const float*, int64_t, const float*, int64_t, int64_t, const int32_t*, int32_t,
                       void*, void*, int, int64_t, int64_t, float*, int32_t*);
int cbxo_nsf_source(const float*, int64_t, int64_t, int32_t, int32_t, const float*, const float*,
                    const float*, float, float*);
int cbxo_hann_window(int32_t, float*);
int cbxo_stft(const float*, int64_t, int64_t, int32_t, int32_t, const float*, int, float*);
int cbxo_istft_post(const float*, int64_t, int64_t, int32_t, int32_t, const float*, int, float,
                    float*);
int cbxo_timestep_embed(const float*, int64_t, const float*, int32_t, float, int, float*);
void cbxo_f32_to_type(const float*, void*, int64_t, int);
void cbxo_type_to_f32(const void*, float*, int64_t, int);
}

namespace {

int g_fail = 0;

uint64_t g_rng = 0x9E3779B97F4A7C15ull;
float uniform() {
    g_rng = g_rng * 6364136223846793005ull + 1442695040888963407ull;
    return (float)((g_rng >> 40) + 0.5) / (float)(1ull << 24);
}
float normal() {  // Box-Muller
    const float u = uniform(), v = uniform();
    return std::sqrt(-2.0f * std::log(u)) * std::cos(6.2831853f * v);
}
std::vector<float> randn(size_t n, float s = 1.0f, float m = 0.0f) {
    std::vector<float> v(n);
    for (auto& x : v) x = m + s * normal();
    return v;
}

template <typename T>
T* to_dev(const std::vector<T>& h) {
    T* d = nullptr;
    cudaMalloc(&d, h.size() * sizeof(T) + 16);
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}
template <typename T>
std::vector<T> to_host(const T* d, size_t n) {
    std::vector<T> h(n);
    cudaDeviceSynchronize();
    cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
}

void check_close(const char* what, const std::vector<float>& got, const std::vector<float>& ref) {
    double worst = 0.0;
    size_t at = 0;
    for (size_t i = 0; i < ref.size(); ++i) {
        const double err = std::fabs((double)got[i] - ref[i]);
        const double bound = 1e-6 + 1e-5 * std::fabs((double)ref[i]);
        if (err / bound > worst) {
            worst = err / bound;
            at = i;
        }
    }
    const bool ok = worst <= 1.0;
    std::printf("%-28s %s (max err/bound %.3f at %zu)\n", what, ok ? "ok" : "FAIL", worst, at);
    if (!ok) ++g_fail;
}

void check(const char* what, bool ok) {
    std::printf("%-28s %s\n", what, ok ? "ok" : "FAIL");
    if (!ok) ++g_fail;
}

}  // namespace

int main() {
    if (cudaSetDevice(0) != cudaSuccess) {
        std::printf("no CUDA device\n");
        return 2;
    }
    // --- add_layer_norm on T3 rows: ne = (1024, 64) ---------------------------
    {
        const int H = 1024, N = 64;
        auto x = randn((size_t)H * N), r = randn((size_t)H * N), w = randn(H, 0.1f, 1.0f),
             b = randn(H, 0.1f);
        float *dx = to_dev(x), *dr = to_dev(r), *dw = to_dev(w), *db = to_dev(b), *ds, *dy;
        cudaMalloc(&ds, x.size() * 4);
        cudaMalloc(&dy, x.size() * 4);
        cbx::Tensor tx = cbx::view(dx, CBX_TYPE_F32, H, N), tr = cbx::view(dr, CBX_TYPE_F32, H, N);
        cbx::Tensor tw = cbx::view(dw, CBX_TYPE_F32, H), tb = cbx::view(db, CBX_TYPE_F32, H);
        cbx::Tensor ts = cbx::view(ds, CBX_TYPE_F32, H, N), ty = cbx::view(dy, CBX_TYPE_F32, H, N);
        check("add_layer_norm returns out", cbx::add_layer_norm(tx, tr, &tw, &tb, 1e-5f, &ts, ty) == &ty);
        std::vector<float> s_ref(x.size()), y_ref(x.size());
        cbxo_add_layernorm_act(x.data(), r.data(), 0, H, w.data(), b.data(), 1e-5f, N, H,
                               s_ref.data(), y_ref.data(), 0, H, 0, nullptr);
        check("add_layer_norm sum exact", to_host(ds, x.size()) == s_ref);
        check_close("add_layer_norm y", to_host(dy, x.size()), y_ref);
        // plain layer_norm (cfm_decoder.cpp:29 helper)
        check("layer_norm returns out", cbx::layer_norm(tx, &tw, &tb, 1e-5f, ty) == &ty);
        cbxo_add_layernorm_act(x.data(), nullptr, 0, H, w.data(), b.data(), 1e-5f, N, H, nullptr,
                               y_ref.data(), 0, H, 0, nullptr);
        check_close("layer_norm y", to_host(dy, x.size()), y_ref);
        // error behaviour: a view whose dim-2 stride breaks the row spacing
        cbx::Tensor bad = cbx::view(dx, CBX_TYPE_F32, H, N / 2, 2);
        bad.nb[2] += 16;
        check("layer_norm bad view -> null", cbx::layer_norm(bad, &tw, &tb, 1e-5f, ty) == nullptr);
        cudaFree(dx); cudaFree(dr); cudaFree(dw); cudaFree(db); cudaFree(ds); cudaFree(dy);
    }
    // --- causal_block1d tail on the engine layout ne = (C=256, T=50, B=2) -------
    {
        const int C = 256, T = 50, B = 2;
        auto x = randn((size_t)C * T * B, 2.0f, 0.5f), w = randn(C, 0.1f, 1.0f), b = randn(C, 0.1f);
        std::vector<float> mask((size_t)T * B, 1.0f);
        for (int t = 40; t < T; ++t) mask[T + t] = 0.0f;
        float *dx = to_dev(x), *dw = to_dev(w), *db = to_dev(b), *dm = to_dev(mask), *dy;
        cudaMalloc(&dy, x.size() * 4);
        cbx::Tensor tx = cbx::view(dx, CBX_TYPE_F32, C, T, B), ty = cbx::view(dy, CBX_TYPE_F32, C, T, B);
        cbx::Tensor tw = cbx::view(dw, CBX_TYPE_F32, C), tb = cbx::view(db, CBX_TYPE_F32, C);
        cbx::Tensor tm = cbx::view(dm, CBX_TYPE_F32, T, B);
        check("layer_norm_mish_mask out", cbx::layer_norm_mish_mask(tx, &tw, &tb, &tm, 1e-5f, ty) == &ty);
        std::vector<float> ref(x.size());
        cbxo_layernorm_channels(x.data(), w.data(), b.data(), 1e-5f, mask.data(), B, C, T, 1, 1,
                                ref.data());
        check_close("layer_norm_mish_mask y", to_host(dy, x.size()), ref);
        cudaFree(dx); cudaFree(dw); cudaFree(db); cudaFree(dm); cudaFree(dy);
    }
    // --- causal conv epilogue + block tail: y_TC ne = (T=64, C=256, B=2) -> (C, T, B) --
    {
        const int C = 256, T = 64, B = 2;
        auto x = randn((size_t)C * T * B, 2.0f), cb = randn(C, 0.5f);
        auto w = randn(C, 0.1f, 1.0f), b = randn(C, 0.1f);
        std::vector<float> mask((size_t)T * B, 1.0f);
        for (int t = 50; t < T; ++t) mask[T + t] = 0.0f;
        float *dx = to_dev(x), *dcb = to_dev(cb), *dw = to_dev(w), *db = to_dev(b);
        float *dm = to_dev(mask), *dy;
        cudaMalloc(&dy, x.size() * 4);
        cbx::Tensor tx = cbx::view(dx, CBX_TYPE_F32, T, C, B), ty = cbx::view(dy, CBX_TYPE_F32, C, T, B);
        cbx::Tensor tcb = cbx::view(dcb, CBX_TYPE_F32, C), tw = cbx::view(dw, CBX_TYPE_F32, C);
        cbx::Tensor tb = cbx::view(db, CBX_TYPE_F32, C), tm = cbx::view(dm, CBX_TYPE_F32, T, B);
        check("conv_bias_layer_norm_mish_mask out",
              cbx::conv_bias_layer_norm_mish_mask(tx, &tcb, &tw, &tb, &tm, 1e-5f, ty) == &ty);
        // reference: bias per channel row, transpose to [B][T][C], LN over C + Mish + mask
        std::vector<float> h((size_t)C * T * B), ref(h.size());
        for (int bb = 0; bb < B; ++bb)
            for (int c = 0; c < C; ++c)
                for (int t = 0; t < T; ++t)
                    h[((size_t)bb * T + t) * C + c] = x[((size_t)bb * C + c) * T + t] + cb[c];
        cbxo_layernorm_channels(h.data(), w.data(), b.data(), 1e-5f, mask.data(), B, C, T, 1, 1,
                                ref.data());
        check_close("conv_bias_layer_norm_mish_mask y", to_host(dy, x.size()), ref);
        cbx::Tensor wrong = cbx::view(dy, CBX_TYPE_F32, T, C, B);  // (T, C) out: rejected
        check("conv_bias_layer_norm_mish_mask bad out -> null",
              cbx::conv_bias_layer_norm_mish_mask(tx, &tcb, &tw, &tb, &tm, 1e-5f, wrong) == nullptr);
        cudaFree(dx); cudaFree(dcb); cudaFree(dw); cudaFree(db); cudaFree(dm); cudaFree(dy);
    }
    // --- snake on ne = (C=64, T=300, B=2), alpha_inv formed on the device -------
    {
        const int C = 64, T = 300, B = 2;
        auto x = randn((size_t)C * T * B);
        std::vector<float> a(C);
        for (auto& v : a) v = std::exp(0.3f * normal());
        float *dx = to_dev(x), *da = to_dev(a), *dy;
        cudaMalloc(&dy, x.size() * 4);
        cbx::Tensor tx = cbx::view(dx, CBX_TYPE_F32, C, T, B), ty = cbx::view(dy, CBX_TYPE_F32, C, T, B);
        cbx::Tensor ta = cbx::view(da, CBX_TYPE_F32, C);
        check("snake out", cbx::snake(tx, ta, nullptr, ty) == &ty);
        std::vector<float> ref(x.size());
        cbxo_snake(x.data(), a.data(), nullptr, 1e-9f, B, C, T, 1, ref.data());
        check_close("snake y", to_host(dy, x.size()), ref);
        cudaFree(dx); cudaFree(da); cudaFree(dy);
    }
    // --- gelu / mish ------------------------------------------------------------
    {
        auto x = randn(1000, 4.0f);
        float *dx = to_dev(x), *dy;
        cudaMalloc(&dy, x.size() * 4);
        cbx::Tensor tx = cbx::view(dx, CBX_TYPE_F32, 1000), ty = cbx::view(dy, CBX_TYPE_F32, 1000);
        std::vector<float> ref(x.size());
        cbx::gelu(tx, ty);
        cbxo_gelu_tanh(x.data(), ref.data(), 1000, 0);
        check_close("gelu", to_host(dy, x.size()), ref);
        cbx::mish(tx, ty);
        cbxo_mish(x.data(), ref.data(), 1000, 0);
        check_close("mish", to_host(dy, x.size()), ref);
        cudaFree(dx); cudaFree(dy);
    }
    // --- get_rows_add: f16 tables -> f32 out, positions n_past + i (bit-exact) ---
    {
        const int H = 64, V = 97, P = 50, N = 19, n_past = 7;
        auto tok32 = randn((size_t)V * H, 0.02f), pos32 = randn((size_t)P * H, 0.02f);
        std::vector<uint16_t> tok(tok32.size()), pos(pos32.size());
        cbxo_f32_to_type(tok32.data(), tok.data(), (int64_t)tok.size(), 1);
        cbxo_f32_to_type(pos32.data(), pos.data(), (int64_t)pos.size(), 1);
        std::vector<int32_t> ids(N);
        for (int i = 0; i < N; ++i) ids[i] = (i * 37 + 5) % V;
        uint16_t *dt = to_dev(tok), *dp = to_dev(pos);
        int32_t* di = to_dev(ids);
        float* dout;
        cudaMalloc(&dout, (size_t)N * H * 4);
        cbx::Tensor tt = cbx::view(dt, CBX_TYPE_F16, H, V), tp = cbx::view(dp, CBX_TYPE_F16, H, P);
        cbx::Tensor ti = cbx::view(di, CBX_TYPE_F32, N);
        ti.nb[0] = 4;  // int32 ids (type is not consulted for ids)
        cbx::Tensor to = cbx::view(dout, CBX_TYPE_F32, H, N);
        check("get_rows_add out", cbx::get_rows_add(tt, ti, &tp, nullptr, n_past, to) == &to);
        std::vector<float> ref((size_t)N * H);
        int32_t err = 0;
        cbxo_embed_gather_add(tok.data(), 1, V, pos.data(), 1, P, ids.data(), nullptr, n_past, N, H,
                              ref.data(), 0, &err);
        check("get_rows_add bit-exact", to_host(dout, ref.size()) == ref && err == 0);
        cudaFree(dt); cudaFree(dp); cudaFree(di); cudaFree(dout);
    }
    // --- get_rows_add_batched: 3 utterances x 17 tokens at positions n_past + t (bit-exact) ---
    {
        const int H = 64, V = 97, P = 50, B = 3, T = 17, n_past = 5;
        auto tok32 = randn((size_t)V * H, 0.02f), pos32 = randn((size_t)P * H, 0.02f);
        std::vector<uint16_t> tok(tok32.size()), pos(pos32.size());
        cbxo_f32_to_type(tok32.data(), tok.data(), (int64_t)tok.size(), 1);
        cbxo_f32_to_type(pos32.data(), pos.data(), (int64_t)pos.size(), 1);
        std::vector<int32_t> ids(B * T), pids(B * T);
        for (int i = 0; i < B * T; ++i) {
            ids[i] = (i * 29 + 3) % V;
            pids[i] = n_past + i % T;
        }
        uint16_t *dt = to_dev(tok), *dp = to_dev(pos);
        int32_t* di = to_dev(ids);
        float* dout;
        cudaMalloc(&dout, (size_t)B * T * H * 4);
        cbx::Tensor tt = cbx::view(dt, CBX_TYPE_F16, H, V), tp = cbx::view(dp, CBX_TYPE_F16, H, P);
        cbx::Tensor ti = cbx::view(di, CBX_TYPE_F32, T, B);
        ti.nb[0] = 4;
        cbx::Tensor to = cbx::view(dout, CBX_TYPE_F32, H, T, B);
        check("get_rows_add_batched out",
              cbx::get_rows_add_batched(tt, ti, &tp, n_past, to) == &to);
        std::vector<float> ref((size_t)B * T * H);
        int32_t err = 0;
        cbxo_embed_gather_add(tok.data(), 1, V, pos.data(), 1, P, ids.data(), pids.data(), 0, B * T,
                              H, ref.data(), 0, &err);
        check("get_rows_add_batched exact", to_host(dout, ref.size()) == ref && err == 0);
        cudaFree(dt); cudaFree(dp); cudaFree(di); cudaFree(dout);
    }
    // --- t3_prefill_input: [cond ; speech[prompt] ; text[tokens]] + pos (bit-exact) ---
    {
        const int H = 64, S = 97, Vt = 130, P = 80, NP = 11, NT = 23, n_past = 3;
        auto sp32 = randn((size_t)S * H, 0.02f), tx32 = randn((size_t)Vt * H, 0.02f);
        auto pos32 = randn((size_t)P * H, 0.02f), cond = randn(H);
        std::vector<uint16_t> sp(sp32.size()), tx(tx32.size()), pos(pos32.size());
        cbxo_f32_to_type(sp32.data(), sp.data(), (int64_t)sp.size(), 1);
        cbxo_f32_to_type(tx32.data(), tx.data(), (int64_t)tx.size(), 1);
        cbxo_f32_to_type(pos32.data(), pos.data(), (int64_t)pos.size(), 1);
        std::vector<int32_t> pr(NP), tk(NT);
        for (int i = 0; i < NP; ++i) pr[i] = (i * 13 + 2) % S;
        for (int i = 0; i < NT; ++i) tk[i] = (i * 29 + 7) % Vt;
        uint16_t *dsp = to_dev(sp), *dtx = to_dev(tx), *dpos = to_dev(pos);
        int32_t *dpr = to_dev(pr), *dtk = to_dev(tk);
        float* dc = to_dev(cond);
        const int N = 1 + NP + NT;
        float* dout;
        cudaMalloc(&dout, (size_t)N * H * 4);
        cbx::Tensor tsp = cbx::view(dsp, CBX_TYPE_F16, H, S), ttx = cbx::view(dtx, CBX_TYPE_F16, H, Vt);
        cbx::Tensor tpos = cbx::view(dpos, CBX_TYPE_F16, H, P), tc = cbx::view(dc, CBX_TYPE_F32, H);
        cbx::Tensor tpr = cbx::view(dpr, CBX_TYPE_F32, NP), ttk = cbx::view(dtk, CBX_TYPE_F32, NT);
        tpr.nb[0] = ttk.nb[0] = 4;  // int32 ids
        cbx::Tensor to = cbx::view(dout, CBX_TYPE_F32, H, N);
        check("t3_prefill_input out",
              cbx::t3_prefill_input(&tc, tsp, &tpr, ttx, ttk, tpos, n_past, to) == &to);
        // the engine's composition: cond row + pos, then the two gathers at their offsets
        std::vector<float> ref((size_t)N * H);
        std::vector<float> posf(pos.size());
        cbxo_type_to_f32(pos.data(), posf.data(), (int64_t)pos.size(), 1);
        for (int j = 0; j < H; ++j) ref[j] = cond[j] + posf[(size_t)n_past * H + j];
        int32_t err = 0;
        cbxo_embed_gather_add(sp.data(), 1, S, pos.data(), 1, P, pr.data(), nullptr, n_past + 1, NP,
                              H, ref.data() + H, 0, &err);
        cbxo_embed_gather_add(tx.data(), 1, Vt, pos.data(), 1, P, tk.data(), nullptr,
                              n_past + 1 + NP, NT, H, ref.data() + (size_t)(1 + NP) * H, 0, &err);
        check("t3_prefill_input bit-exact", to_host(dout, ref.size()) == ref && err == 0);
        cudaFree(dsp); cudaFree(dtx); cudaFree(dpos); cudaFree(dpr); cudaFree(dtk); cudaFree(dc);
        cudaFree(dout);
    }
    // --- sinusoidal_pos_emb (+ SiLU), dim 320, scale 1000 -------------------------
    {
        const int dim = 320, n = 8;
        std::vector<float> t(n), fr(dim / 2);
        for (auto& v : t) v = uniform();
        check("cbx_sinusoid_freqs", cbx_sinusoid_freqs(dim, fr.data()) == CBX_OK);
        std::vector<float> fr_ref(dim / 2);
        cbxo_sinusoid_freqs(dim, fr_ref.data());
        check("freqs equal the engine's", fr == fr_ref);
        float *dt = to_dev(t), *df = to_dev(fr), *dy;
        cudaMalloc(&dy, (size_t)n * dim * 4);
        cbx::Tensor tt = cbx::view(dt, CBX_TYPE_F32, n), tf = cbx::view(df, CBX_TYPE_F32, dim / 2);
        cbx::Tensor ty = cbx::view(dy, CBX_TYPE_F32, dim, n);
        check("sinusoidal_pos_emb out", cbx::sinusoidal_pos_emb(tt, dim, 1000.0f, tf, true, ty) == &ty);
        std::vector<float> ref((size_t)n * dim);
        cbxo_timestep_embed(t.data(), n, fr.data(), dim, 1000.0f, 2, ref.data());
        check_close("sinusoidal_pos_emb+silu", to_host(dy, ref.size()), ref);
        cudaFree(dt); cudaFree(df); cudaFree(dy);
    }
    // --- GEMM-epilogue neighbours -------------------------------------------------
    {
        const int H = 512, N = 12;
        auto x = randn((size_t)H * N, 3.0f), b = randn(H, 0.5f), cb = randn(N);
        float *dx = to_dev(x), *db = to_dev(b), *dcb = to_dev(cb), *dy;
        cudaMalloc(&dy, x.size() * 4);
        cbx::Tensor tx = cbx::view(dx, CBX_TYPE_F32, H, N), ty = cbx::view(dy, CBX_TYPE_F32, H, N);
        cbx::Tensor tb = cbx::view(db, CBX_TYPE_F32, H), tcb = cbx::view(dcb, CBX_TYPE_F32, N);
        std::vector<float> ref(x.size());
        cbx::add_bias_act(tx, &tb, false, CBX_ACT_GELU_TANH, 0.0f, ty);
        cbxo_bias_act(x.data(), ref.data(), 0, N, H, b.data(), 0, H, 3, 0.0f);
        check_close("add_bias_act fc+gelu", to_host(dy, x.size()), ref);
        cbx::add_bias_act(tx, &tcb, true, CBX_ACT_NONE, 0.0f, ty);
        cbxo_bias_act(x.data(), ref.data(), 0, N, H, cb.data(), 1, N, 0, 0.0f);
        check("add_bias_act per-row exact", to_host(dy, x.size()) == ref);
        cbx::leaky_relu(tx, 0.1f, ty);
        cbxo_bias_act(x.data(), ref.data(), 0, N, H, nullptr, 0, 0, 5, 0.1f);
        check_close("leaky_relu", to_host(dy, x.size()), ref);
        cbx::elu(tx, ty);
        cbxo_bias_act(x.data(), ref.data(), 0, N, H, nullptr, 0, 0, 6, 0.0f);
        check_close("elu", to_host(dy, x.size()), ref);
        cbx::gelu_erf(tx, ty);
        cbxo_gelu_erf(x.data(), ref.data(), (int64_t)x.size(), 0);
        check_close("gelu_erf", to_host(dy, x.size()), ref);
        std::vector<float> g = to_host(dy, x.size());  // the third input, as on the device
        cbx::sum3_scale(tx, tx, ty, 1.0f / 3.0f, ty);   // in place on the third input
        cbxo_sum3_scale(x.data(), x.data(), g.data(), 1.0f / 3.0f, ref.data(), (int64_t)x.size(), 0);
        check("sum3_scale exact", to_host(dy, x.size()) == ref);
        cudaFree(dx); cudaFree(db); cudaFree(dcb); cudaFree(dy);
    }
    // --- T3 QKV epilogue: prefill chunk and one token per stream ------------------
    {
        const int D = 64, N = 5, ctx = 12;
        auto h = randn((size_t)N * 3 * D), b = randn(3 * D, 0.1f);
        std::vector<int32_t> pos = {3, 11, 0, 7, 12};  // the last is out of range
        float *dh = to_dev(h), *db = to_dev(b), *dq, *dk, *dv;
        int32_t *dpos = to_dev(pos), *derr;
        cudaMalloc(&dq, (size_t)N * D * 4);
        cudaMalloc(&dk, (size_t)N * ctx * D * 4);
        cudaMalloc(&dv, (size_t)N * ctx * D * 4);
        cudaMalloc(&derr, 4);
        cudaMemset(dk, 0, (size_t)N * ctx * D * 4);
        cudaMemset(dv, 0, (size_t)N * ctx * D * 4);
        cudaMemset(derr, 0, 4);
        cbx::Tensor tq = cbx::view(dh, CBX_TYPE_F32, 3 * D, N), tb = cbx::view(db, CBX_TYPE_F32, 3 * D);
        cbx::Tensor tk = cbx::view(dk, CBX_TYPE_F32, D, ctx, N), tv = cbx::view(dv, CBX_TYPE_F32, D, ctx, N);
        cbx::Tensor tp = cbx::view(dpos, CBX_TYPE_F32, N), to = cbx::view(dq, CBX_TYPE_F32, D, N);
        check("qkv_kv_append out",
              cbx::qkv_kv_append(tq, &tb, tk, tv, &tp, 0, (int64_t)ctx * D, ctx, &to, derr) == &to);
        std::vector<float> rq((size_t)N * D), rk((size_t)N * ctx * D, 0.f), rv = rk;
        int32_t rerr = 0;
        cbxo_qkv_kv_append(h.data(), 3 * D, b.data(), N, D, pos.data(), 0, rk.data(), rv.data(), 0,
                           (int64_t)ctx * D, ctx, rq.data(), &rerr);
        check("qkv_kv_append q exact", to_host(dq, rq.size()) == rq);
        check("qkv_kv_append k/v exact",
              to_host(dk, rk.size()) == rk && to_host(dv, rv.size()) == rv);
        check("qkv_kv_append oob flagged", to_host(derr, 1)[0] == rerr && rerr == CBX_EFLAG_POS_OOB);
        cudaFree(dh); cudaFree(db); cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dpos); cudaFree(derr);
    }
    // --- HiFT: the engine's draws, generate_source, STFT, iSTFT tail -------------
    {
        const int n_mel = 6, up = 480, T = n_mel * up, B = 1;
        std::vector<float> f0 = {0.f, 120.f, 180.5f, 95.f, 0.f, 210.f};
        std::vector<float> ph(9), nz((size_t)9 * T), ph2(9), nz2((size_t)9 * T);
        cbx::engine_source_draws(42, T, nullptr, ph.data(), nz.data());
        cbx::engine_source_draws(42, T, nullptr, ph2.data(), nz2.data());
        check("engine draws repeatable", ph == ph2 && nz == nz2 && ph[0] == 0.0f);
        std::vector<float> lw = randn(9, 0.4f);
        float *df0 = to_dev(f0), *dph = to_dev(ph), *dnz = to_dev(nz), *dsrc;
        cudaMalloc(&dsrc, (size_t)T * 4);
        cbx::Tensor tf0 = cbx::view(df0, CBX_TYPE_F32, n_mel, B), tph = cbx::view(dph, CBX_TYPE_F32, 9, B);
        cbx::Tensor tnz = cbx::view(dnz, CBX_TYPE_F32, T, 9, B), tsrc = cbx::view(dsrc, CBX_TYPE_F32, T, B);
        check("generate_source out",
              cbx::generate_source(tf0, tph, tnz, lw.data(), 0.05f, up, 24000, tsrc) == &tsrc);
        std::vector<float> rsrc(T);
        cbxo_nsf_source(f0.data(), B, n_mel, up, 24000, ph.data(), nz.data(), lw.data(), 0.05f,
                        rsrc.data());
        check_close("generate_source y", to_host(dsrc, rsrc.size()), rsrc);
        std::vector<float> win(16);
        cbx_hann_window(16, win.data());
        float* dw = to_dev(win);
        cbx::Tensor tw = cbx::view(dw, CBX_TYPE_F32, 16);
        const int Ts = T / 4 + 1;
        float* dsp;
        cudaMalloc(&dsp, (size_t)Ts * 18 * 4);
        cbx::Tensor tsp = cbx::view(dsp, CBX_TYPE_F32, 18, Ts, B);
        check("stft_centered out", cbx::stft_centered(tsrc, tw, 16, 4, tsp) == &tsp);
        std::vector<float> rsp((size_t)Ts * 18), src_gpu = to_host(dsrc, T);
        cbxo_stft(src_gpu.data(), B, T, 16, 4, win.data(), 1, rsp.data());
        check_close("stft_centered y", to_host(dsp, rsp.size()), rsp);
        // output tail on a synthetic conv_post block (18 channels per frame)
        const int Tf = 200;
        auto post = randn((size_t)Tf * 18, 1.0f, -1.0f);
        float *dpost = to_dev(post), *dwav;
        cudaMalloc(&dwav, (size_t)(Tf - 1) * 4 * 4);
        cbx::Tensor tpost = cbx::view(dpost, CBX_TYPE_F32, 18, Tf, B);
        cbx::Tensor twav = cbx::view(dwav, CBX_TYPE_F32, (Tf - 1) * 4, B);
        check("istft_post out", cbx::istft_post(tpost, tw, 16, 4, 0.99f, twav) == &twav);
        std::vector<float> rwav((size_t)(Tf - 1) * 4);
        cbxo_istft_post(post.data(), B, Tf, 16, 4, win.data(), 1, 0.99f, rwav.data());
        check_close("istft_post y", to_host(dwav, rwav.size()), rwav);
        cudaFree(df0); cudaFree(dph); cudaFree(dnz); cudaFree(dsrc); cudaFree(dw); cudaFree(dsp);
        cudaFree(dpost); cudaFree(dwav);
    }
    const cudaError_t e = cudaDeviceSynchronize();
    check("no CUDA error", e == cudaSuccess);
    std::printf("%s: %d failure(s)\n", g_fail ? "FAILED" : "PASSED", g_fail);
    return g_fail ? 1 : 0;
}
