// cbx_layer_helpers.hpp — C++ host mirror of chatterbox-cpp's layer helpers on
// top of the libcbx_ops C ABI (cbx_ops.h).  Header-only.
//
// The engine builds these ops as ggml graph nodes from static helpers
// (layer_norm / mish / snake / sinusoidal_pos_emb / the inline T3 code).  The
// functions below keep those helpers' names and argument meanings, but take
// a ggml-like tensor view of device memory and enqueue one libcbx_ops kernel
// on a CUDA stream instead of emitting nodes:
//
//   cbx::layer_norm          cfm_decoder.cpp:29-33, flow_encoder.cpp:58-62
//   cbx::add_layer_norm      t3.cpp:528-532 (attn_residual = cur + h; LN2)
//   cbx::mish                cfm_decoder.cpp:36-38
//   cbx::gelu / cbx::silu    t3.cpp:537 / cfm_decoder.cpp:466
//   cbx::gelu_erf            cfm_decoder.cpp:239, s3enc.cpp:177
//   cbx::add_bias_act        t3.cpp:536-537 (fc bias + gelu), cfm_decoder.cpp:114
//   cbx::elu / leaky_relu    hift_vocoder.cpp:575 / :686, :748
//   cbx::sum3_scale          hift_vocoder.cpp:733-739 (ResBlock average)
//   cbx::layer_norm_mish_mask  causal_block1d tail, cfm_decoder.cpp:144-148
//   cbx::snake               hift_vocoder.cpp:64-73
//   cbx::sinusoidal_pos_emb  cfm_decoder.cpp:49-62 (batched, on the device)
//   cbx::get_rows_add        t3.cpp:440-455 (+ positions n_past + i, :597-600)
//   cbx::get_rows_add_batched  the same for B utterances at positions n_past + t
//   cbx::t3_prefill_input    t3.cpp:428-455 ([cond ; speech[prompt] ; tokens] + positions)
//   cbx::qkv_kv_append       t3.cpp:465-489 (qkv bias, Q, K / V cache writes)
//   cbx::generate_source     hift_vocoder.cpp:853-965 (HiFTVocoder::generate_source)
//   cbx::engine_source_draws hift_vocoder.cpp:889-913 (its std::mt19937 draws, host)
//   cbx::stft_centered       hift_vocoder.cpp:465-498 (+ s_stft rows, :627-638)
//   cbx::istft_post          hift_vocoder.cpp:787-829 (magnitude / phase, iSTFT, clamp)
//
// Tensors follow ggml: ne[0] is innermost, nb[] are byte strides, `type` is a
// cbx_type (== ggml_type).  Outputs are caller-allocated views.  Error
// behaviour follows the engine: on failure a helper prints
// "<helper>: <message>" to stderr and returns nullptr (cf. t3.cpp:353-371);
// on success it returns a pointer to `out`.
#ifndef CBX_LAYER_HELPERS_HPP
#define CBX_LAYER_HELPERS_HPP

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <random>

#include "cbx_ops.h"

namespace cbx {

struct Tensor {
    int type = CBX_TYPE_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    size_t nb[4] = {0, 0, 0, 0};
    void* data = nullptr;  // device pointer
};

inline size_t type_size(int type) { return type == CBX_TYPE_F32 ? 4 : 2; }

// Contiguous view of `data` with shape ne0 x ne1 x ne2 x ne3 (ggml order).
inline Tensor view(void* data, int type, int64_t ne0, int64_t ne1 = 1, int64_t ne2 = 1,
                   int64_t ne3 = 1) {
    Tensor t;
    t.type = type;
    t.data = data;
    t.ne[0] = ne0;
    t.ne[1] = ne1;
    t.ne[2] = ne2;
    t.ne[3] = ne3;
    t.nb[0] = type_size(type);
    for (int i = 1; i < 4; ++i) t.nb[i] = t.nb[i - 1] * (size_t)t.ne[i - 1];
    return t;
}

inline int64_t nelements(const Tensor& t) { return t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]; }
inline int64_t nrows(const Tensor& t) { return t.ne[1] * t.ne[2] * t.ne[3]; }

namespace detail {
inline Tensor* report(const char* helper, int status, Tensor* out) {
    if (status == CBX_OK) return out;
    std::fprintf(stderr, "%s: %s (%s)\n", helper, cbx_last_error(), cbx_status_string(status));
    return nullptr;
}
inline bool contiguous(const Tensor& t) {
    size_t s = type_size(t.type);
    for (int i = 0; i < 4; ++i) {
        if (t.nb[i] != s) return false;
        s *= (size_t)t.ne[i];
    }
    return true;
}
// Rows of ne[0] elements equally spaced by nb[1] (dims 2, 3 folded into rows).
inline bool uniform_rows(const Tensor& t, int64_t* stride_elems) {
    const size_t s = type_size(t.type);
    if (t.nb[0] != s || t.nb[1] % s) return false;
    if (t.nb[2] != t.nb[1] * (size_t)t.ne[1] || t.nb[3] != t.nb[2] * (size_t)t.ne[2]) return false;
    *stride_elems = (int64_t)(t.nb[1] / s);
    return true;
}
inline const float* f32_or_null(const Tensor* t) {
    return t ? static_cast<const float*>(t->data) : nullptr;
}
}  // namespace detail

// y = LN(x) * w + b over ne0 (w, b f32 [ne0] or null).
inline Tensor* layer_norm(const Tensor& x, const Tensor* w, const Tensor* b, float eps,
                          Tensor& out, cbx_stream_t stream = nullptr) {
    int64_t sx = 0, so = 0;
    if (!detail::uniform_rows(x, &sx) || !detail::uniform_rows(out, &so)) {
        std::fprintf(stderr, "layer_norm: x / out must be rows with a uniform stride\n");
        return nullptr;
    }
    return detail::report("layer_norm",
                          cbx_add_layernorm(x.data, nullptr, x.type, sx, detail::f32_or_null(w),
                                            detail::f32_or_null(b), eps, nrows(x), x.ne[0],
                                            nullptr, out.data, out.type, so, stream),
                          &out);
}

// sum = x + resid (written to *sum_out when given); out = LN(sum) * w + b.
inline Tensor* add_layer_norm(const Tensor& x, const Tensor& resid, const Tensor* w,
                              const Tensor* b, float eps, Tensor* sum_out, Tensor& out,
                              cbx_stream_t stream = nullptr) {
    int64_t sx = 0, sr = 0, so = 0, ss = 0;
    if (!detail::uniform_rows(x, &sx) || !detail::uniform_rows(resid, &sr) || sr != sx ||
        !detail::uniform_rows(out, &so) ||
        (sum_out && (!detail::uniform_rows(*sum_out, &ss) || ss != so))) {
        std::fprintf(stderr, "add_layer_norm: x/resid and sum_out/out need matching row strides\n");
        return nullptr;
    }
    return detail::report(
        "add_layer_norm",
        cbx_add_layernorm(x.data, resid.data, x.type, sx, detail::f32_or_null(w),
                          detail::f32_or_null(b), eps, nrows(x), x.ne[0],
                          sum_out ? sum_out->data : nullptr, out.data, out.type, so, stream),
        &out);
}

namespace detail {
template <int (*F)(const void*, void*, int64_t, int, cbx_stream_t)>
inline Tensor* unary(const char* name, const Tensor& x, Tensor& out, cbx_stream_t stream) {
    if (!contiguous(x) || !contiguous(out) || x.type != out.type ||
        nelements(x) != nelements(out)) {
        std::fprintf(stderr, "%s: x and out must be contiguous with equal type and size\n", name);
        return nullptr;
    }
    return report(name, F(x.data, out.data, nelements(x), x.type, stream), &out);
}
}  // namespace detail

inline Tensor* mish(const Tensor& x, Tensor& out, cbx_stream_t stream = nullptr) {
    return detail::unary<cbx_mish>("mish", x, out, stream);
}
inline Tensor* gelu(const Tensor& x, Tensor& out, cbx_stream_t stream = nullptr) {
    return detail::unary<cbx_gelu_tanh>("gelu", x, out, stream);
}
inline Tensor* silu(const Tensor& x, Tensor& out, cbx_stream_t stream = nullptr) {
    return detail::unary<cbx_silu>("silu", x, out, stream);
}
// ggml_gelu_erf (cfm_decoder.cpp:239, s3enc.cpp:177)
inline Tensor* gelu_erf(const Tensor& x, Tensor& out, cbx_stream_t stream = nullptr) {
    return detail::unary<cbx_gelu_erf>("gelu_erf", x, out, stream);
}

// act(x + bias): bias f32 ne = (ne0) added along ne0 (t3.cpp:536-537, fc bias then
// gelu), or, with per_row, ne = (C) added per row of a (T, C) tensor
// (add_bias_TC, cfm_decoder.cpp:114).  bias may be null (plain activation).
inline Tensor* add_bias_act(const Tensor& x, const Tensor* bias, bool per_row, int act,
                            float act_param, Tensor& out, cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(x) || !detail::contiguous(out) || x.type != out.type) {
        std::fprintf(stderr, "add_bias_act: contiguous x / out of one type required\n");
        return nullptr;
    }
    return detail::report(
        "add_bias_act",
        cbx_bias_act(x.data, out.data, x.type, nrows(x), x.ne[0], detail::f32_or_null(bias),
                     per_row ? CBX_BIAS_NE1 : CBX_BIAS_NE0, bias ? nelements(*bias) : 0, act,
                     act_param, stream),
        &out);
}
// ggml_elu (hift_vocoder.cpp:575) / ggml_leaky_relu (hift_vocoder.cpp:686, :748)
inline Tensor* elu(const Tensor& x, Tensor& out, cbx_stream_t stream = nullptr) {
    return add_bias_act(x, nullptr, false, CBX_ACT_ELU, 0.0f, out, stream);
}
inline Tensor* leaky_relu(const Tensor& x, float slope, Tensor& out, cbx_stream_t stream = nullptr) {
    return add_bias_act(x, nullptr, false, CBX_ACT_LEAKY_RELU, slope, out, stream);
}

// ((a + b) + c) * scale: the HiFT ResBlock average (hift_vocoder.cpp:733-739).
inline Tensor* sum3_scale(const Tensor& a, const Tensor& b, const Tensor& c, float scale,
                          Tensor& out, cbx_stream_t stream = nullptr) {
    if (nelements(a) != nelements(out) || nelements(b) != nelements(a) ||
        nelements(c) != nelements(a)) {
        std::fprintf(stderr, "sum3_scale: sizes differ\n");
        return nullptr;
    }
    return detail::report("sum3_scale",
                          cbx_sum3_scale(a.data, b.data, c.data, scale, out.data, nelements(a),
                                         a.type, stream),
                          &out);
}

// causal_block1d tail on the engine layout x ne = (C, T[, B]) f32:
// out = mish(LN_C(x) * w + b) * mask[t] (mask f32 ne = (T[, B]) or null).
inline Tensor* layer_norm_mish_mask(const Tensor& x_CT, const Tensor* w, const Tensor* b,
                                    const Tensor* mask_T, float eps, Tensor& out,
                                    cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(x_CT) || !detail::contiguous(out) || x_CT.type != CBX_TYPE_F32 ||
        out.type != CBX_TYPE_F32) {
        std::fprintf(stderr, "layer_norm_mish_mask: contiguous f32 (C, T) tensors required\n");
        return nullptr;
    }
    return detail::report(
        "layer_norm_mish_mask",
        cbx_layernorm_channels(static_cast<const float*>(x_CT.data), detail::f32_or_null(w),
                               detail::f32_or_null(b), eps, detail::f32_or_null(mask_T),
                               x_CT.ne[2] * x_CT.ne[3], x_CT.ne[0], x_CT.ne[1], CBX_LAYOUT_BTC,
                               CBX_ACT_MISH, static_cast<float*>(out.data), stream),
        &out);
}

// causal_conv1d's epilogue + causal_block1d tail: the conv GEMM output
// y_TC ne = (T, C[, B]) f32 (before add_bias_TC) -> out ne = (C, T[, B]) =
// mish(LN_C(y_TC^T + conv_b) * w + b) * mask[t], replacing add_bias_TC,
// ggml_cont(ggml_transpose), layer_norm, mish and the mask multiply.
inline Tensor* conv_bias_layer_norm_mish_mask(const Tensor& y_TC, const Tensor* conv_b,
                                              const Tensor* w, const Tensor* b,
                                              const Tensor* mask_T, float eps, Tensor& out,
                                              cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(y_TC) || !detail::contiguous(out) || y_TC.type != CBX_TYPE_F32 ||
        out.type != CBX_TYPE_F32 || out.ne[0] != y_TC.ne[1] || out.ne[1] != y_TC.ne[0]) {
        std::fprintf(stderr,
                     "conv_bias_layer_norm_mish_mask: contiguous f32 (T, C) in, (C, T) out\n");
        return nullptr;
    }
    return detail::report(
        "conv_bias_layer_norm_mish_mask",
        cbx_causal_block1d_tail(static_cast<const float*>(y_TC.data), detail::f32_or_null(conv_b),
                                detail::f32_or_null(w), detail::f32_or_null(b), eps,
                                detail::f32_or_null(mask_T), y_TC.ne[2] * y_TC.ne[3], y_TC.ne[1],
                                y_TC.ne[0], CBX_ACT_MISH, static_cast<float*>(out.data), stream),
        &out);
}

// snake(ctx, x, alpha, alpha_inv) on the engine layout x ne = (C, T[, B]) f32;
// alpha / alpha_inv f32 ne = (C); alpha_inv null = 1 / (alpha + 1e-9).
inline Tensor* snake(const Tensor& x, const Tensor& alpha, const Tensor* alpha_inv, Tensor& out,
                     cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(x) || !detail::contiguous(out) || x.type != CBX_TYPE_F32 ||
        alpha.ne[0] != x.ne[0]) {
        std::fprintf(stderr, "snake: contiguous f32 x (C, T) and alpha (C) required\n");
        return nullptr;
    }
    return detail::report(
        "snake",
        cbx_snake(static_cast<const float*>(x.data), static_cast<const float*>(alpha.data),
                  detail::f32_or_null(alpha_inv), 1e-9f, x.ne[2] * x.ne[3], x.ne[0], x.ne[1],
                  CBX_LAYOUT_BTC, static_cast<float*>(out.data), stream),
        &out);
}

// Batched sinusoidal_pos_emb: out ne = (dim, n_t) f32; t f32 ne = (n_t);
// freqs f32 ne = (dim / 2) from cbx_sinusoid_freqs (uploaded once).
inline Tensor* sinusoidal_pos_emb(const Tensor& t, int dim, float scale, const Tensor& freqs,
                                  bool then_silu, Tensor& out, cbx_stream_t stream = nullptr) {
    return detail::report(
        "sinusoidal_pos_emb",
        cbx_timestep_embed(static_cast<const float*>(t.data), nelements(t),
                           static_cast<const float*>(freqs.data), dim, scale,
                           then_silu ? CBX_ACT_SILU : CBX_ACT_NONE,
                           static_cast<float*>(out.data), stream),
        &out);
}

// T3 embedding: out[i] = tok_table[ids[i]] + pos_table[pos_ids ? pos_ids[i] : n_past + i].
// Tables ne = (H, rows); ids / pos_ids int32 ne = (N); out ne = (H, N).
inline Tensor* get_rows_add(const Tensor& tok_table, const Tensor& ids, const Tensor* pos_table,
                            const Tensor* pos_ids, int64_t n_past, Tensor& out,
                            int32_t* err_word = nullptr, cbx_stream_t stream = nullptr) {
    return detail::report(
        "get_rows_add",
        cbx_embed_gather_add(tok_table.data, tok_table.type, tok_table.ne[1],
                             pos_table ? pos_table->data : nullptr,
                             pos_table ? pos_table->type : CBX_TYPE_F32,
                             pos_table ? pos_table->ne[1] : 0,
                             static_cast<const int32_t*>(ids.data),
                             pos_ids ? static_cast<const int32_t*>(pos_ids->data) : nullptr, n_past,
                             nelements(ids), tok_table.ne[0], out.data, out.type, err_word, stream),
        &out);
}

// The gather of B utterances prefilled together, each at positions n_past ..
// n_past + T - 1 (t3.cpp:440-455 per utterance): ids int32 ne = (T, B),
// out ne = (H, T, B), out[b][t] = tok_table[ids[b][t]] + pos_table[n_past + t].
inline Tensor* get_rows_add_batched(const Tensor& tok_table, const Tensor& ids,
                                    const Tensor* pos_table, int64_t n_past, Tensor& out,
                                    int32_t* err_word = nullptr, cbx_stream_t stream = nullptr) {
    return detail::report(
        "get_rows_add_batched",
        cbx_embed_gather_add_batched(tok_table.data, tok_table.type, tok_table.ne[1],
                                     pos_table ? pos_table->data : nullptr,
                                     pos_table ? pos_table->type : CBX_TYPE_F32,
                                     pos_table ? pos_table->ne[1] : 0,
                                     static_cast<const int32_t*>(ids.data), ids.ne[1], ids.ne[0],
                                     n_past, tok_table.ne[0], out.data, out.type, err_word, stream),
        &out);
}

// T3 prefill input (t3.cpp:428-455): out = [cond_emb ; speech_emb[prompt] ;
// emb_table[tokens]] + pos_embd[n_past + i].  cond_emb f32 ne = (H) or (H, n)
// (the cond_enc GEMM output + bias) or null; prompt / tokens int32 ne = (n);
// prompt may be null (no prompt speech); tables ne = (H, rows); out ne = (H, N).
inline Tensor* t3_prefill_input(const Tensor* cond_emb, const Tensor& speech_emb,
                                const Tensor* prompt, const Tensor& emb_table,
                                const Tensor& tokens, const Tensor& pos_embd, int64_t n_past,
                                Tensor& out, int32_t* err_word = nullptr,
                                cbx_stream_t stream = nullptr) {
    const int64_t H = emb_table.ne[0];
    const int64_t n_cond = cond_emb ? nelements(*cond_emb) / H : 0;
    return detail::report(
        "t3_prefill_input",
        cbx_t3_embed_sequence(cond_emb ? static_cast<const float*>(cond_emb->data) : nullptr, n_cond,
                              speech_emb.data, speech_emb.type, speech_emb.ne[1],
                              prompt ? static_cast<const int32_t*>(prompt->data) : nullptr,
                              prompt ? nelements(*prompt) : 0, emb_table.data, emb_table.type,
                              emb_table.ne[1], static_cast<const int32_t*>(tokens.data),
                              nelements(tokens), pos_embd.data, pos_embd.type, pos_embd.ne[1],
                              n_past, H, out.data, out.type, err_word, stream),
        &out);
}

// T3 QKV epilogue (t3.cpp:465-489).  qkv f32 ne = (3D, N) (the GEMM output
// without bias); qkv_b f32 ne = (3D) or null; cache_k / cache_v: the engine's
// per-stream cache tensors, rows of D elements (f32, or f16 / bf16); q_out f32
// ne = (D, N) or null.  Prefill form: positions null, rows n_past + i of one
// slab.  Batched decode form: positions int32 ne = (N) (each stream's n_past),
// row r in slab r, slab_stride elements apart.  err_word: device int32
// (CBX_EFLAG_POS_OOB for rows past max_context).
inline Tensor* qkv_kv_append(const Tensor& qkv, const Tensor* qkv_b, Tensor& cache_k,
                             Tensor& cache_v, const Tensor* positions, int64_t n_past,
                             int64_t slab_stride, int64_t max_context, Tensor* q_out,
                             int32_t* err_word, cbx_stream_t stream = nullptr) {
    int64_t sx = 0;
    if (qkv.type != CBX_TYPE_F32 || !detail::uniform_rows(qkv, &sx) || qkv.ne[0] % 3 ||
        cache_k.type != cache_v.type) {
        std::fprintf(stderr, "qkv_kv_append: f32 rows of 3D elements and caches of one type\n");
        return nullptr;
    }
    Tensor* ret = q_out ? q_out : &cache_k;
    return detail::report(
        "qkv_kv_append",
        cbx_qkv_kv_append(static_cast<const float*>(qkv.data), sx, detail::f32_or_null(qkv_b),
                          nrows(qkv), qkv.ne[0] / 3,
                          positions ? static_cast<const int32_t*>(positions->data) : nullptr,
                          (int32_t)n_past, cache_k.data, cache_v.data, cache_k.type, slab_stride,
                          max_context, q_out ? static_cast<float*>(q_out->data) : nullptr,
                          err_word, stream),
        ret);
}

// The random inputs HiFTVocoder::generate_source draws when none are given
// (hift_vocoder.cpp:889-913), on the host with the same standard-library
// generators in the same order: std::mt19937(seed); unless phase_opt is given,
// 9 phases from uniform_real_distribution<float>(-pi, pi) with phase[0] = 0;
// then n_wav * 9 normals from normal_distribution<float>(0, 1), harmonic-major
// (noise[h * n_wav + t]).  With the same C++ standard library as the engine the
// draws are identical; upload them and call generate_source.
inline void engine_source_draws(uint64_t seed, int64_t n_wav, const float* phase_opt,
                                float* phase_out, float* noise_out) {
    std::mt19937 rng(static_cast<std::mt19937::result_type>(seed));
    if (phase_opt) {
        for (int h = 0; h < CBX_NSF_HARMONICS; ++h) phase_out[h] = phase_opt[h];
    } else {
        std::uniform_real_distribution<float> u(-3.14159265358979323846f, 3.14159265358979323846f);
        for (int h = 0; h < CBX_NSF_HARMONICS; ++h) phase_out[h] = u(rng);
    }
    phase_out[0] = 0.0f;
    std::normal_distribution<float> n(0.0f, 1.0f);
    for (int64_t i = 0; i < n_wav * CBX_NSF_HARMONICS; ++i) noise_out[i] = n(rng);
}

// HiFTVocoder::generate_source for a batch: f0 f32 ne = (n_mel, B); phase f32
// ne = (9, B); noise f32 ne = (n_mel * upsample, 9, B); lin_w: the 9 l_linear
// weights on the host; out f32 ne = (n_mel * upsample, B).
inline Tensor* generate_source(const Tensor& f0, const Tensor& phase, const Tensor& noise,
                               const float* lin_w, float lin_b, int upsample, int sampling_rate,
                               Tensor& out, cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(f0) || !detail::contiguous(noise) || !detail::contiguous(out) ||
        noise.ne[0] != f0.ne[0] * upsample || out.ne[0] != noise.ne[0]) {
        std::fprintf(stderr, "generate_source: contiguous f0 / noise / out of matching sizes\n");
        return nullptr;
    }
    return detail::report(
        "generate_source",
        cbx_nsf_source(static_cast<const float*>(f0.data), nrows(f0), f0.ne[0], upsample,
                       sampling_rate, static_cast<const float*>(phase.data),
                       static_cast<const float*>(noise.data), lin_w, lin_b,
                       static_cast<float*>(out.data), stream),
        &out);
}

// stft_centered_host + the s_stft rows: audio f32 ne = (T, B); window f32 ne =
// (n_fft); out f32 ne = (2 nb, T / hop + 1, B) (nb real bins then nb imag bins
// per frame, the engine's (T_stft, 18) layout).
inline Tensor* stft_centered(const Tensor& audio, const Tensor& window, int n_fft, int hop,
                             Tensor& out, cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(audio) || !detail::contiguous(out)) {
        std::fprintf(stderr, "stft_centered: contiguous audio / out required\n");
        return nullptr;
    }
    return detail::report(
        "stft_centered",
        cbx_stft(static_cast<const float*>(audio.data), nrows(audio), audio.ne[0], n_fft, hop,
                 static_cast<const float*>(window.data), CBX_LAYOUT_BTC,
                 static_cast<float*>(out.data), stream),
        &out);
}

// The HiFT output tail: post f32 ne = (2 nb, T_final, B) (conv_post's rows);
// out f32 ne = ((T_final - 1) * hop, B), clamped to +-audio_limit.
inline Tensor* istft_post(const Tensor& post, const Tensor& window, int n_fft, int hop,
                          float audio_limit, Tensor& out, cbx_stream_t stream = nullptr) {
    if (!detail::contiguous(post) || !detail::contiguous(out)) {
        std::fprintf(stderr, "istft_post: contiguous post / out required\n");
        return nullptr;
    }
    return detail::report(
        "istft_post",
        cbx_istft_post(static_cast<const float*>(post.data), post.ne[2] * post.ne[3], post.ne[1],
                       n_fft, hop, static_cast<const float*>(window.data), CBX_LAYOUT_BTC,
                       audio_limit, static_cast<float*>(out.data), stream),
        &out);
}

}  // namespace cbx

#endif  // CBX_LAYER_HELPERS_HPP
