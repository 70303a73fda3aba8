/*
 * cbx_oracle.c — CPU restatement of the libcbx_ops hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library
 * and the timed CPU baseline of bench.py; it is never linked into, loaded by
 * or called from the product path (chatterbox_amdvulkan_b200/).
 *
 * What it restates.  The reference engine (tarekedOz/Chatterbox_AMDVulkan,
 * chatterbox-cpp) composes these ops from ggml graph nodes; ggml itself
 * (third_party/ggml, pinned v0.12.0 by chatterbox-cpp/CMakeLists.txt:46) is an
 * empty submodule in the reference checkout, so ggml's CPU kernels cannot be
 * compiled here.  The oracle therefore restates, for each helper:
 *   - the node composition and order of the engine's helper (cited per
 *     function), rounding to f32 at every ggml node boundary, and
 *   - the op formulas of the reference's own NumPy oracles
 *     (scripts/reference_t3_forward.py, reference_cfm_decoder.py,
 *     reference_hift_vocoder.py), with every transcendental evaluated in
 *     double and rounded once to f32, and LayerNorm statistics in double.
 * The sinusoidal embedding is a host C++ loop in the engine
 * (cfm_decoder.cpp:49-62); it is restated with the same f32 libm calls.
 *
 * Parity pin: tests/golden/make_golden.py imports the reference's NumPy
 * oracle functions and writes fixtures that tests/test_oracle_golden.py checks
 * this file against.
 *
 * Element types use ggml_type numbering: 0 = f32, 1 = f16, 30 = bf16.
 * Layouts: 0 = [B][C][T] (T contiguous), 1 = [B][T][C] (C contiguous).
 * Activations: 0 none, 1 mish, 2 silu, 3 gelu-tanh, 4 gelu-erf, 5 leaky relu,
 * 6 elu.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_F32 = 0, T_F16 = 1, T_BF16 = 30 };
enum { L_BCT = 0, L_BTC = 1 };
enum { A_NONE = 0, A_MISH = 1, A_SILU = 2, A_GELU = 3, A_GELU_ERF = 4, A_LEAKY = 5, A_ELU = 6 };

/* ---------------------------------------------------------------- types -- */

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* f32 -> bf16, round to nearest even; NaN stays NaN (quiet). */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

static inline uint16_t f32_to_f16(float f) {
    _Float16 v = (_Float16)f; /* IEEE round to nearest even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline int type_size(int t) { return t == T_F32 ? 4 : 2; }

static inline float load_elt(const void* p, int t, int64_t i) {
    if (t == T_F32) return ((const float*)p)[i];
    if (t == T_BF16) return bf16_to_f32(((const uint16_t*)p)[i]);
    return f16_to_f32(((const uint16_t*)p)[i]);
}

static inline void store_elt(void* p, int t, int64_t i, float v) {
    if (t == T_F32) ((float*)p)[i] = v;
    else if (t == T_BF16) ((uint16_t*)p)[i] = f32_to_bf16(v);
    else ((uint16_t*)p)[i] = f32_to_f16(v);
}

static inline int valid_type(int t) { return t == T_F32 || t == T_F16 || t == T_BF16; }

/* ---------------------------------------------------------- activations -- */

/* GELU-tanh, one ggml_gelu node (chatterbox-cpp/src/t3.cpp:537); formula
 * scripts/reference_t3_forward.py:73-77. */
static inline float gelu_tanh_1(float x) {
    const double xd = x;
    const double u = 0.79788456080286535588 * (xd + 0.044715 * xd * xd * xd);
    /* 0.5 (1 + tanh(u)) = 1 / (1 + e^(-2u)): the same function without the
     * cancellation of 1 + tanh(u) for large negative x */
    return (float)(xd / (1.0 + exp(-2.0 * u)));
}

/* SiLU, one ggml_silu node (cfm_decoder.cpp:466); formula
 * scripts/reference_cfm_decoder.py:141-142. */
static inline float silu_1(float x) {
    const double xd = x;
    return (float)(xd / (1.0 + exp(-xd)));
}

/* Mish = ggml_mul(x, ggml_tanh(ggml_softplus(x))) (cfm_decoder.cpp:36-38):
 * three nodes, each rounded to f32.  Softplus is the identity above 20
 * (scripts/reference_cfm_decoder.py:145-149). */
static inline float mish_1(float x) {
    const double xd = x;
    const float sp = (x > 20.0f) ? x : (float)log1p(exp(xd));
    const float th = (float)tanh((double)sp);
    return x * th;
}

/* Exact GELU, one ggml_gelu_erf node (cfm_decoder.cpp:239, s3enc.cpp:177);
 * formula scripts/reference_cfm_decoder.py:152-155, 0.5 x (1 + erf(x / sqrt 2))
 * evaluated as 0.5 x erfc(-x / sqrt 2) in double. */
static inline float gelu_erf_1(float x) {
    const double xd = x;
    return (float)(0.5 * xd * erfc(-xd * 0.70710678118654752440));
}

/* ELU (alpha 1), ggml_elu (hift_vocoder.cpp:575); scripts/reference_hift_vocoder.py:132-133. */
static inline float elu_1(float x) { return x >= 0.0f ? x : (float)expm1((double)x); }

/* LeakyReLU, ggml_leaky_relu (hift_vocoder.cpp:686, :748);
 * scripts/reference_hift_vocoder.py:136-137: x >= 0 ? x : x * slope in f32. */
static inline float leaky_1(float x, float slope) { return x >= 0.0f ? x : x * slope; }

static inline float act_1(int act, float v) {
    switch (act) {
        case A_MISH: return mish_1(v);
        case A_SILU: return silu_1(v);
        case A_GELU: return gelu_tanh_1(v);
        case A_GELU_ERF: return gelu_erf_1(v);
        case A_ELU: return elu_1(v);
        default: return v;
    }
}

/* -------------------------------------------------------------- threads -- */

int cbxo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

int cbxo_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------ embedding gather-add -- */

/* chatterbox-cpp/src/t3.cpp:440-455: get_rows(tok) -> cast(F32), get_rows(pos)
 * -> cast(F32), add; positions n_past + i filled on the host at t3.cpp:597-600;
 * reference_t3_forward.py:163-170 is the same sum in NumPy.  An id or a
 * position out of range zeroes the row and sets the matching error bit. */
int cbxo_embed_gather_add(const void* tok, int tok_t, int64_t n_tok,
                          const void* pos, int pos_t, int64_t n_pos,
                          const int32_t* ids, const int32_t* pos_ids, int64_t pos_offset,
                          int64_t n_rows, int64_t hidden, void* out, int out_t, int32_t* err) {
    if (!tok || !ids || !out || n_rows < 0 || hidden <= 0) return -1;
    if (!valid_type(tok_t) || !valid_type(out_t) || (pos && !valid_type(pos_t))) return -2;
    int32_t flags = 0;
#pragma omp parallel for schedule(static) reduction(| : flags)
    for (int64_t i = 0; i < n_rows; ++i) {
        const int64_t id = ids[i];
        const int64_t p = pos_ids ? (int64_t)pos_ids[i] : pos_offset + i;
        int bad = 0;
        if (id < 0 || id >= n_tok) { bad = 1; flags |= 1; }
        if (pos && (p < 0 || p >= n_pos)) { bad = 1; flags |= 2; }
        for (int64_t j = 0; j < hidden; ++j) {
            float v = 0.0f;
            if (!bad) {
                v = load_elt(tok, tok_t, id * hidden + j);
                if (pos) v = v + load_elt(pos, pos_t, p * hidden + j);
            }
            store_elt(out, out_t, i * hidden + j, v);
        }
    }
    if (err) *err |= flags;
    return 0;
}

/* ------------------------------------------ residual-add + LayerNorm -- */

/* Row LayerNorm of one f32 row `s` into `yrow` (f32 scratch):
 * ggml_norm (mean/biased variance, chatterbox-cpp/src/t3.cpp:465,
 * reference_t3_forward.py:80-84) then ggml_mul(gamma), ggml_add(beta), each
 * rounded to f32. */
static void ln_row(const float* s, int64_t H, const float* g, const float* b, float eps,
                   float* yrow) {
    double sum = 0.0;
    for (int64_t j = 0; j < H; ++j) sum += s[j];
    const double mean = sum / (double)H;
    double ss = 0.0;
    for (int64_t j = 0; j < H; ++j) {
        const double d = (double)s[j] - mean;
        ss += d * d;
    }
    const double var = ss / (double)H;
    const double rstd = 1.0 / sqrt(var + (double)eps);
    for (int64_t j = 0; j < H; ++j) {
        float n = (float)(((double)s[j] - mean) * rstd); /* ggml_norm */
        if (g) n = n * g[j];                              /* ggml_mul  */
        if (b) n = n + b[j];                              /* ggml_add  */
        yrow[j] = n;
    }
}

/* chatterbox-cpp/src/t3.cpp:528-532 (attn_residual = cur + h; LN2) and
 * :541 + :465-466 (h = cur + attn_residual; next LN1); resid == NULL is the
 * plain layer_norm() helper (cfm_decoder.cpp:29-33, flow_encoder.cpp:58-62).
 * act / mask extend it to the engine-native [T][C] CausalBlock1D tail
 * (cfm_decoder.cpp:144-148): y = act(LN(s)) * mask[row]. */
int cbxo_add_layernorm_act(const void* x, const void* r, int in_t, int64_t in_stride,
                           const float* g, const float* b, float eps,
                           int64_t n_rows, int64_t H,
                           void* s_out, void* y, int out_t, int64_t out_stride,
                           int act, const float* mask) {
    if (!x || !y || n_rows < 0 || H <= 0) return -1;
    if (!valid_type(in_t) || !valid_type(out_t)) return -2;
    if (in_stride == 0) in_stride = H;
    if (out_stride == 0) out_stride = H;
#pragma omp parallel
    {
        float* srow = (float*)__builtin_alloca((size_t)H * sizeof(float));
        float* yrow = (float*)__builtin_alloca((size_t)H * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t i = 0; i < n_rows; ++i) {
            for (int64_t j = 0; j < H; ++j) {
                float v = load_elt(x, in_t, i * in_stride + j);
                if (r) v = v + load_elt(r, in_t, i * in_stride + j); /* ggml_add */
                srow[j] = v;
            }
            ln_row(srow, H, g, b, eps, yrow);
            const float m = mask ? mask[i] : 1.0f;
            for (int64_t j = 0; j < H; ++j) {
                float v = act_1(act, yrow[j]);
                if (mask) v = v * m;
                if (s_out) store_elt(s_out, in_t, i * out_stride + j, srow[j]);
                store_elt(y, out_t, i * out_stride + j, v);
            }
        }
    }
    return 0;
}

int cbxo_add_layernorm(const void* x, const void* r, int in_t, int64_t in_stride,
                       const float* g, const float* b, float eps, int64_t n_rows, int64_t H,
                       void* s_out, void* y, int out_t, int64_t out_stride) {
    return cbxo_add_layernorm_act(x, r, in_t, in_stride, g, b, eps, n_rows, H, s_out, y, out_t,
                                  out_stride, A_NONE, NULL);
}

/* -------------------------------------- LayerNorm over C (+act, +mask) -- */

/* CausalBlock1D tail, chatterbox-cpp/src/cfm_decoder.cpp:144-148:
 * layer_norm over C (:29-33), mish (:36-38), * mask (:148).  BCT is the
 * PyTorch layout of scripts/reference_cfm_decoder.py:241-256 (transpose to
 * [B,T,C], LN, transpose back, Mish, mask). */
int cbxo_layernorm_channels(const float* x, const float* g, const float* b, float eps,
                            const float* mask, int64_t B, int64_t C, int64_t T, int layout,
                            int act, float* y) {
    if (!x || !y || B < 0 || C <= 0 || T < 0) return -1;
    if (layout != L_BCT && layout != L_BTC) return -1;
    if (layout == L_BTC)
        return cbxo_add_layernorm_act(x, NULL, T_F32, C, g, b, eps, B * T, C, NULL, y, T_F32, C,
                                      act, mask);
#pragma omp parallel
    {
        float* col = (float*)__builtin_alloca((size_t)C * sizeof(float));
        float* yc = (float*)__builtin_alloca((size_t)C * sizeof(float));
#pragma omp for schedule(static)
        for (int64_t bt = 0; bt < B * T; ++bt) {
            const int64_t bi = bt / T, t = bt % T;
            const float* xb = x + bi * C * T;
            for (int64_t c = 0; c < C; ++c) col[c] = xb[c * T + t];
            ln_row(col, C, g, b, eps, yc);
            const float m = mask ? mask[bi * T + t] : 1.0f;
            for (int64_t c = 0; c < C; ++c) {
                float v = act_1(act, yc[c]);
                if (mask) v = v * m;
                y[bi * C * T + c * T + t] = v;
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------- elementwise -- */

static int unary(int act, const void* x, void* y, int64_t n, int t) {
    if (!x || !y || n < 0) return -1;
    if (!valid_type(t)) return -2;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) store_elt(y, t, i, act_1(act, load_elt(x, t, i)));
    return 0;
}

int cbxo_gelu_tanh(const void* x, void* y, int64_t n, int t) { return unary(A_GELU, x, y, n, t); }
int cbxo_gelu_erf(const void* x, void* y, int64_t n, int t) { return unary(A_GELU_ERF, x, y, n, t); }
int cbxo_silu(const void* x, void* y, int64_t n, int t) { return unary(A_SILU, x, y, n, t); }
int cbxo_mish(const void* x, void* y, int64_t n, int t) { return unary(A_MISH, x, y, n, t); }

/* ------------------------------------------------ epilogue neighbours -- */

/* y[r, j] = act(x[r, j] + b): ggml_add (rounded to f32) then the activation
 * node.  Bias along ne0 (bias[j]: t3.cpp:536-537 fc bias then ggml_gelu) or
 * along ne1 (bias[r % bias_len]: add_bias_TC, cfm_decoder.cpp:114); no bias:
 * the plain activation (hift_vocoder.cpp:575 elu, :686 / :748 leaky_relu). */
int cbxo_bias_act(const void* x, void* y, int t, int64_t n_rows, int64_t H, const float* bias,
                  int axis, int64_t bias_len, int act, float param) {
    if (!x || !y || n_rows < 0 || H <= 0 || act < 0 || act > A_ELU) return -1;
    if (axis != 0 && axis != 1) return -1;
    if (bias && ((axis == 0 && bias_len != H) || (axis == 1 && bias_len <= 0))) return -1;
    if (!valid_type(t)) return -2;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n_rows; ++r) {
        for (int64_t j = 0; j < H; ++j) {
            float v = load_elt(x, t, r * H + j);
            if (bias) v = v + (axis == 0 ? bias[j] : bias[r % bias_len]); /* ggml_add */
            v = (act == A_LEAKY) ? leaky_1(v, param) : act_1(act, v);
            store_elt(y, t, r * H + j, v);
        }
    }
    return 0;
}

/* hift_vocoder.cpp:733-739: sum = r0; sum = add(sum, r1); sum = add(sum, r2);
 * x = scale(sum, 1/3) — three f32 nodes in that order. */
int cbxo_sum3_scale(const void* a, const void* b, const void* c, float scale, void* y, int64_t n,
                    int t) {
    if (!a || !b || !c || !y || n < 0) return -1;
    if (!valid_type(t)) return -2;
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < n; ++e) {
        float v = load_elt(a, t, e) + load_elt(b, t, e);
        v = v + load_elt(c, t, e);
        store_elt(y, t, e, v * scale);
    }
    return 0;
}

/* ----------------------------------------------- sinusoidal embedding -- */

/* chatterbox-cpp/src/cfm_decoder.cpp:52-56: f32 log/exp exactly as the engine
 * writes them (std::log / std::exp on float = logf / expf). */
int cbxo_sinusoid_freqs(int32_t dim, float* freqs) {
    if (!freqs || dim < 4) return -1;
    const int half = dim / 2;
    const float log10000 = logf(10000.0f);
    const float factor = log10000 / (float)(half - 1);
    for (int j = 0; j < half; ++j) freqs[j] = expf(-factor * (float)j);
    return 0;
}

/* chatterbox-cpp/src/cfm_decoder.cpp:57-60 for a batch of t, then the SiLU
 * of the time MLP (:466) when act == silu.  a = (scale * t) * div in f32. */
int cbxo_timestep_embed(const float* t, int64_t n_t, const float* freqs, int32_t dim, float scale,
                        int act, float* y) {
    if (!t || !freqs || !y || n_t < 0 || dim < 4) return -1;
    if (act != A_NONE && act != A_SILU) return -1;
    const int half = dim / 2;
    for (int64_t i = 0; i < n_t; ++i) {
        const float st = scale * t[i];
        float* yi = y + i * dim;
        for (int j = 0; j < half; ++j) {
            const float a = st * freqs[j];
            yi[j] = sinf(a);
            yi[j + half] = cosf(a);
        }
        if (dim & 1) yi[dim - 1] = 0.0f;
        if (act == A_SILU)
            for (int j = 0; j < dim; ++j) yi[j] = silu_1(yi[j]);
    }
    return 0;
}

/* --------------------------------------------------------------- snake -- */

/* hift_vocoder.cpp:419-420: 1 / (alpha + eps) in f32. */
int cbxo_snake_alpha_inv(const float* alpha, int64_t n, float eps, float* inv) {
    if (!alpha || !inv || n < 0) return -1;
    for (int64_t i = 0; i < n; ++i) inv[i] = 1.0f / (alpha[i] + eps);
    return 0;
}

/* chatterbox-cpp/src/hift_vocoder.cpp:64-73: xa = x*alpha; s = sin(xa);
 * s2 = s*s; m = s2*alpha_inv; y = x + m — five ggml nodes, each rounded to
 * f32 (scripts/reference_hift_vocoder.py:140-145 is the same formula). */
static inline float snake_1(float x, float a, float ainv) {
    const float xa = x * a;
    const float s = (float)sin((double)xa);
    const float s2 = s * s;
    const float m = s2 * ainv;
    return x + m;
}

int cbxo_snake(const float* x, const float* alpha, const float* alpha_inv, float eps, int64_t B,
               int64_t C, int64_t T, int layout, float* y) {
    if (!x || !alpha || !y || B < 0 || C <= 0 || T < 0) return -1;
    if (layout != L_BCT && layout != L_BTC) return -1;
    const int64_t n = B * C * T;
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < n; ++e) {
        const int64_t c = (layout == L_BCT) ? (e / T) % C : e % C;
        const float a = alpha[c];
        const float ainv = alpha_inv ? alpha_inv[c] : 1.0f / (a + eps);
        y[e] = snake_1(x[e], a, ainv);
    }
    return 0;
}

/* ------------------------------------------------ QKV epilogue + KV cache -- */

/* chatterbox-cpp/src/t3.cpp:465-489: cur = ggml_add(mul_mat(qkv_w, x), qkv_b)
 * (f32), Q = cont(view rows [0, D)), ggml_cpy of rows [D, 2D) and [2D, 3D)
 * into cache_k / cache_v at position n_past + i (converted to the cache type).
 * Rows generalise to one token per stream: position positions[r] (NULL:
 * pos_offset + r) in slab r (slab_stride elements apart).  Out-of-range
 * positions write nothing and set bit 2 of *err. */
int cbxo_qkv_kv_append(const float* qkv, int64_t stride, const float* bias, int64_t n_rows,
                       int64_t D, const int32_t* positions, int32_t pos_offset, void* ck, void* cv,
                       int ct, int64_t slab_stride, int64_t max_context, float* q, int32_t* err) {
    if (!qkv || !ck || !cv || n_rows < 0 || D <= 0 || !valid_type(ct) || max_context <= 0)
        return -1;
    if (stride == 0) stride = 3 * D;
    int32_t e = 0;
    for (int64_t r = 0; r < n_rows; ++r) {
        const float* row = qkv + r * stride;
        const int64_t pos = positions ? positions[r] : pos_offset + r;
        const int ok = pos >= 0 && pos < max_context;
        if (!ok) e |= 2;
        for (int64_t i = 0; i < D; ++i) {
            const float tq = row[i] + (bias ? bias[i] : 0.0f);
            const float tk = row[D + i] + (bias ? bias[D + i] : 0.0f);
            const float tv = row[2 * D + i] + (bias ? bias[2 * D + i] : 0.0f);
            if (q) q[r * D + i] = tq;
            if (ok) {
                store_elt(ck, ct, r * slab_stride + pos * D + i, tk);
                store_elt(cv, ct, r * slab_stride + pos * D + i, tv);
            }
        }
    }
    if (err) *err |= e;
    return 0;
}

/* ------------------------------------------- HiFT source and STFT/iSTFT -- */

enum { NSF_HARM = 9 };  /* NB_HARMONICS + 1, hift_vocoder.cpp:858-862 */

/* HiFTVocoder::generate_source, chatterbox-cpp/src/hift_vocoder.cpp:853-965,
 * with the phase and noise arrays given (its phase_vec_opt / noise_z_opt form;
 * phase[b][0] is forced to 0 as at :885).  Per utterance b and wave sample t:
 * nearest-upsampled f0, voiced mask f > 10, a double running sum per harmonic
 * of f*(h+1)/sr in sample order (:925-934), theta = 2 pi frac(cs) + phase,
 * sine = 0.1f * (float)sin(theta), sine*u + noise_amp*noise, then the 9 -> 1
 * linear merge accumulated in double from f32 products and tanh (:955-963).
 * f0 [B][n_mel], phase [B][9], noise [B][9][T], out [B][T], T = n_mel*upsample. */
int cbxo_nsf_source(const float* f0, int64_t B, int64_t n_mel, int32_t upsample, int32_t sr,
                    const float* phase, const float* noise, const float* lw, float lb,
                    float* out) {
    if (!f0 || !phase || !noise || !lw || !out || B < 0 || n_mel < 0 || upsample <= 0 || sr <= 0)
        return -1;
    const int64_t T = n_mel * upsample;
    const double inv_sr = 1.0 / (double)sr;
    const double two_pi = 2.0 * 3.14159265358979323846;
    const float sine_amp = 0.1f, noise_std = 0.003f, voiced_thr = 10.0f;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b) {
        double cs[NSF_HARM];
        float ph[NSF_HARM];
        for (int h = 0; h < NSF_HARM; ++h) {
            cs[h] = 0.0;
            ph[h] = h == 0 ? 0.0f : phase[b * NSF_HARM + h];
        }
        for (int64_t t = 0; t < T; ++t) {
            const float f = f0[b * n_mel + t / upsample];
            const float u = (f > voiced_thr) ? 1.0f : 0.0f;
            const float noise_amp = u * noise_std + (1.0f - u) * (sine_amp / 3.0f);
            double s = (double)lb;
            for (int h = 0; h < NSF_HARM; ++h) {
                const double f_h = (double)f * (h + 1) * inv_sr;
                cs[h] += f_h;
                const double frac = cs[h] - floor(cs[h]);
                const double th = two_pi * frac + ph[h];
                const float sine = sine_amp * (float)sin(th);
                const float nz = noise_amp * noise[(b * NSF_HARM + h) * T + t];
                const float sth = sine * u + nz;
                s += lw[h] * sth;
            }
            out[b * T + t] = (float)tanh((double)(float)s);
        }
    }
    return 0;
}

/* Periodic Hann window, the engine's f32 host expression
 * (hift_vocoder.cpp:429-434): 0.5f - 0.5f * cosf(2.0f * (float)pi * n / N). */
int cbxo_hann_window(int32_t n_fft, float* w) {
    if (!w || n_fft <= 0) return -1;
    for (int32_t n = 0; n < n_fft; ++n)
        w[n] = 0.5f - 0.5f * cosf(2.0f * (float)3.14159265358979323846 * n / n_fft);
    return 0;
}

/* Centered STFT, stft_centered_host (hift_vocoder.cpp:465-498): reflect-pad by
 * n_fft/2 (mirror axis = the edge sample), frames every hop samples, frame[n] =
 * x*window in f32, naive DFT in double with the engine's twiddle expression,
 * each bin rounded to f32.  T_stft = 1 + T/hop (n_fft even).  Layout BTC:
 * out[b][t][k] = real, out[b][t][nb + k] = imag (the engine's s_stft rows,
 * :627-638); BCT: out[b][k][t], out[b][nb + k][t]
 * (scripts/reference_hift_vocoder.py:394-395). */
int cbxo_stft(const float* audio, int64_t B, int64_t T, int32_t n_fft, int32_t hop,
              const float* window, int layout, float* out) {
    if (!audio || !window || !out || B < 0 || n_fft < 2 || n_fft > 256 || (n_fft & 1) || hop <= 0)
        return -1;
    if (layout != L_BCT && layout != L_BTC) return -1;
    const int pad = n_fft / 2;
    if (T <= pad) return -1;
    const int64_t Ts = 1 + (T + 2 * pad - n_fft) / hop;
    const int nb = n_fft / 2 + 1;
#pragma omp parallel for schedule(static)
    for (int64_t bt = 0; bt < B * Ts; ++bt) {
        const int64_t b = bt / Ts, t = bt % Ts;
        const float* x = audio + b * T;
        float frame[256];
        for (int n = 0; n < n_fft; ++n) {
            const int64_t i = t * hop + n;  /* index into the padded signal */
            float v;
            if (i < pad) v = x[pad - i];
            else if (i >= pad + T) v = x[T - 2 - (i - pad - T)];
            else v = x[i - pad];
            frame[n] = v * window[n];
        }
        for (int k = 0; k < nb; ++k) {
            double sr = 0.0, si = 0.0;
            for (int n = 0; n < n_fft; ++n) {
                const double a = -2.0 * 3.14159265358979323846 * k * n / n_fft;
                sr += frame[n] * cos(a);
                si += frame[n] * sin(a);
            }
            if (layout == L_BTC) {
                out[(b * Ts + t) * 2 * nb + k] = (float)sr;
                out[(b * Ts + t) * 2 * nb + nb + k] = (float)si;
            } else {
                out[(b * 2 * nb + k) * Ts + t] = (float)sr;
                out[(b * 2 * nb + nb + k) * Ts + t] = (float)si;
            }
        }
    }
    return 0;
}

/* The HiFT output tail, hift_vocoder.cpp:787-829: from conv_post's 2*nb
 * channels, magnitude = min(exp(raw), 100) and phase = sin(raw) per bin,
 * real = mag*cos(phase), imag = mag*sin(phase) in f32; then
 * istft_centered_host (:501-541): per frame a naive inverse DFT in double
 * (DC, 2 Re(X_k e^{+i..}) for 0 < k < nb-1, Nyquist (-1)^n), divided by
 * n_fft and rounded to f32, windowed overlap-add in f32 in frame order with the
 * window-square sum, division where that sum > 1e-11, the n_fft/2 trim, and
 * std::clamp to +-audio_limit.  post layout BTC: [b][t][2 nb] (the engine's
 * (T_final, 18) rows); BCT: [b][2 nb][t].  out [B][(n_frames-1)*hop]. */
int cbxo_istft_post(const float* post, int64_t B, int64_t n_frames, int32_t n_fft, int32_t hop,
                    const float* window, int layout, float audio_limit, float* out) {
    if (!post || !window || !out || B < 0 || n_frames < 1 || n_fft < 2 || n_fft > 256 || (n_fft & 1) ||
        hop <= 0 || hop > n_fft)
        return -1;
    if (layout != L_BCT && layout != L_BTC) return -1;
    const int nb = n_fft / 2 + 1, pad = n_fft / 2;
    const int64_t len = (n_frames - 1) * hop + n_fft;
    const int64_t Ta = len - 2 * pad;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b) {
        float* apad = (float*)calloc((size_t)len, sizeof(float));
        float* wsum = (float*)calloc((size_t)len, sizeof(float));
        float re[129], im[129], frame[256];
        for (int64_t t = 0; t < n_frames; ++t) {
            for (int k = 0; k < nb; ++k) {
                const float mraw = layout == L_BTC ? post[(b * n_frames + t) * 2 * nb + k]
                                                   : post[(b * 2 * nb + k) * n_frames + t];
                const float praw = layout == L_BTC ? post[(b * n_frames + t) * 2 * nb + nb + k]
                                                   : post[(b * 2 * nb + nb + k) * n_frames + t];
                const float e = (float)exp((double)mraw);
                const float mag = (100.0f < e) ? 100.0f : e;     /* std::min(e, 100.0f) */
                const float phs = (float)sin((double)praw);
                re[k] = mag * (float)cos((double)phs);
                im[k] = mag * (float)sin((double)phs);
            }
            for (int n = 0; n < n_fft; ++n) {
                double s = re[0];
                for (int k = 1; k < nb - 1; ++k) {
                    const double a = 2.0 * 3.14159265358979323846 * k * n / n_fft;
                    s += 2.0 * (re[k] * cos(a) - im[k] * sin(a));
                }
                s += re[nb - 1] * ((n & 1) ? -1.0 : 1.0);
                frame[n] = (float)(s / n_fft);
            }
            for (int n = 0; n < n_fft; ++n) {
                apad[t * hop + n] += frame[n] * window[n];
                wsum[t * hop + n] += window[n] * window[n];
            }
        }
        for (int64_t i = 0; i < Ta; ++i) {
            float v = apad[pad + i];
            if (wsum[pad + i] > 1e-11f) v /= wsum[pad + i];
            /* std::clamp(v, -lim, lim) */
            out[b * Ta + i] = (v < -audio_limit) ? -audio_limit : ((audio_limit < v) ? audio_limit : v);
        }
        free(apad);
        free(wsum);
    }
    return 0;
}

/* --------------------------------------------------- dtype round trips -- */

/* Exposed so the tests can pin the conversions against NumPy. */
void cbxo_f32_to_type(const float* in, void* out, int64_t n, int t) {
    for (int64_t i = 0; i < n; ++i) store_elt(out, t, i, in[i]);
}
void cbxo_type_to_f32(const void* in, float* out, int64_t n, int t) {
    for (int64_t i = 0; i < n; ++i) out[i] = load_elt(in, t, i);
}
int cbxo_type_size(int t) { return valid_type(t) ? type_size(t) : -1; }
