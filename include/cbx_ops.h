/*
 * cbx_ops.h — C ABI of libcbx_ops, the B200 (sm_100a) implementation of the
 * fused per-layer elementwise ops that the Chatterbox TTS engine runs between
 * its GEMMs (T3 embedding gather-add, residual-add + LayerNorm, GELU-tanh,
 * SiLU, Mish, channel-strided LayerNorm + Mish for the CFM estimator, the
 * sinusoidal timestep embedding and HiFT's Snake).
 *
 * Each entry point replaces one layer helper of chatterbox-cpp (or the chain
 * of ggml graph nodes it emits); the citation above each declaration names the
 * helper and the ggml ops it composes (paths are relative to the
 * tarekedOz/Chatterbox_AMDVulkan project root).
 *
 * Conventions (shared by every entry point):
 *   - Tensors follow the ggml convention: ne0 is the innermost (contiguous)
 *     dimension, so a "[n_rows][hidden]" buffer is ggml ne = (hidden, n_rows).
 *     Per-channel vectors (gamma, beta, alpha) broadcast along ne0 exactly like
 *     ggml_mul / ggml_add do in the helpers.
 *   - All data pointers are DEVICE pointers owned by the caller.  Nothing on
 *     the compute path allocates, frees or copies to/from the host.  The only
 *     host-side entry points are the table builders marked "host".
 *   - Work is enqueued on the caller's CUDA stream (`cbx_stream_t` is the same
 *     pointer type as cudaStream_t / CUstream).  Device selection is the
 *     caller's cudaSetDevice.  Calls are stateless and reentrant; they may be
 *     made from several host threads on different streams or devices.
 *   - The library keeps small per-device caches (SM count, occupancy, the
 *     kernels' shared-memory opt-in) for the life of the device's primary
 *     context.  Do not use it across a cudaDeviceReset (or a destroyed and
 *     re-created primary context) in the same process.
 *   - Out-of-place or in-place: an output may alias the input it is computed
 *     from (same pointer, same strides, same dtype).  Partial overlaps are not
 *     supported.
 *   - Return value: CBX_OK (0) or a negative cbx_status.  Arguments are
 *     validated on the host before anything is launched; on error nothing is
 *     launched and cbx_last_error() returns a message for the calling thread
 *     (the convention of chatterbox-cpp/src/chatterbox_capi.cpp:14-18,159-161).
 *   - Kernels are launched with programmatic dependent launch enabled, so a
 *     kernel's launch overlaps the tail of the previous kernel in the stream;
 *     every kernel waits for its predecessor before touching global memory, so
 *     stream ordering is unchanged.  Set CBX_DISABLE_PDL=1 to launch plainly.
 */
#ifndef CBX_OPS_H
#define CBX_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define CBX_API __declspec(dllexport)
#else
#define CBX_API __attribute__((visibility("default")))
#endif

typedef struct CUstream_st* cbx_stream_t; /* == cudaStream_t; NULL = legacy default stream */

/* Status codes. */
typedef enum cbx_status {
    CBX_OK                    = 0,
    CBX_ERR_INVALID_ARG       = -1, /* null pointer, bad size/stride/layout/act */
    CBX_ERR_UNSUPPORTED_DTYPE = -2, /* dtype (combination) not implemented      */
    CBX_ERR_LAUNCH            = -3, /* CUDA launch failed (message has the CUDA error) */
    CBX_ERR_INDEX_OOB         = -4, /* reserved: reported through the device error word */
    CBX_ERR_TIMEOUT           = -5, /* a bounded wait gave up                      */
    CBX_ERR_CUDA              = -6  /* other CUDA runtime error                    */
} cbx_status;

/* Element types.  The numeric values are ggml_type's (GGML_TYPE_F32 = 0,
 * GGML_TYPE_F16 = 1, GGML_TYPE_BF16 = 30), so an engine adapter can pass
 * tensor->type straight through. */
typedef enum cbx_type {
    CBX_TYPE_F32  = 0,
    CBX_TYPE_F16  = 1,
    CBX_TYPE_BF16 = 30
} cbx_type;

/* Memory layout of a 3-D activation with batch B, channels C, time T. */
typedef enum cbx_layout {
    CBX_LAYOUT_BCT = 0, /* PyTorch channels-first [B][C][T]: T contiguous        */
    CBX_LAYOUT_BTC = 1  /* engine-native ggml ne=(C,T,B), i.e. [B][T][C]: C contiguous */
} cbx_layout;

/* Activation fused after a normalisation / embedding / bias add.  The
 * normalisation entry points accept NONE..GELU_TANH; cbx_bias_act accepts all. */
typedef enum cbx_act {
    CBX_ACT_NONE       = 0,
    CBX_ACT_MISH       = 1,
    CBX_ACT_SILU       = 2,
    CBX_ACT_GELU_TANH  = 3,
    CBX_ACT_GELU_ERF   = 4, /* 0.5 x (1 + erf(x / sqrt 2))                    */
    CBX_ACT_LEAKY_RELU = 5, /* x >= 0 ? x : slope x   (slope = act_param)     */
    CBX_ACT_ELU        = 6  /* x >= 0 ? x : e^x - 1                          */
} cbx_act;

/* Axis a bias vector broadcasts along (cbx_bias_act). */
typedef enum cbx_bias_axis {
    CBX_BIAS_NE0 = 0, /* bias[j], j < hidden: ggml_add(x, b) with b ne = (hidden)        */
    CBX_BIAS_NE1 = 1  /* bias[r % bias_len]: ggml_add(x, reshape(b, 1, C)) on (T, C)  */
} cbx_bias_axis;

/* Bits of the optional device error word of cbx_embed_gather_add. */
#define CBX_EFLAG_TOKEN_OOB 0x1
#define CBX_EFLAG_POS_OOB   0x2

/* Bits of the library's own device error word (see cbx_device_errors). */
#define CBX_DEVERR_WAIT_TIMEOUT 0x1 /* a bounded wait on a TMA transfer gave up */
#define CBX_DEVERR_SMEM_ALIGN   0x2 /* a staging buffer broke its alignment rule: no output */

/* Library version as (major << 16) | (minor << 8) | patch. */
CBX_API int cbx_version(void);

/* Message for the last failing call on this thread ("" if none). */
CBX_API const char* cbx_last_error(void);

/* Static name of a status code. */
CBX_API const char* cbx_status_string(int status);

/* Reads and clears the library's device error word on the current device:
 * the OR of CBX_DEVERR_* bits raised by kernels since the last call.  Kernels
 * that wait on asynchronous copies bound every wait; one that gives up sets
 * CBX_DEVERR_WAIT_TIMEOUT, leaves its output incomplete and exits instead of
 * hanging the GPU; one whose shared staging buffer is not aligned as its
 * swizzled TMA stores require sets CBX_DEVERR_SMEM_ALIGN and writes nothing.
 * Enqueued on `stream` and synchronises it.  Returns CBX_OK,
 * or CBX_ERR_TIMEOUT when any bit was set (*flags receives the bits; may be
 * NULL).  No counterpart in the reference (ggml reports no device faults). */
CBX_API int cbx_device_errors(int32_t* flags, cbx_stream_t stream);

/* Diagnostic of the bounded-wait machinery: enqueues a one-thread kernel that
 * waits, with the same bounded loop the TMA kernels use but at most `polls`
 * polls (1 .. 2^24), on an mbarrier that nothing completes, and so raises
 * CBX_DEVERR_WAIT_TIMEOUT; cbx_device_errors then reports CBX_ERR_TIMEOUT.
 * No copy is issued and nothing faults.  No counterpart in the reference. */
CBX_API int cbx_selftest_wait_timeout(uint32_t polls, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Token + learned-position embedding gather-add.
 *
 *   out[i, :] = tok_table[ids[i], :] + pos_table[p_i, :],
 *   p_i = pos_ids ? pos_ids[i] : pos_offset + i
 *
 * Both gathered rows are widened to f32, added in f32 and rounded once to
 * out_type, so the result is bit-exact with get_rows → cast(F32) → add.
 * Replaces chatterbox-cpp/src/t3.cpp:440-455 (ggml_get_rows ×2, ggml_cast ×2,
 * ggml_concat, ggml_add) and the host fill of positions at t3.cpp:597-600
 * (pos_ids == NULL with pos_offset = n_past).  pos_table may be NULL for a
 * plain ggml_get_rows (flow_encoder.cpp:588).
 *
 * tok_type, pos_type, out_type: any of F32 / F16 / BF16.
 * An id outside [0, n_tok_rows) or a position outside [0, n_pos_rows) makes
 * the whole output row zero and ORs CBX_EFLAG_TOKEN_OOB / CBX_EFLAG_POS_OOB
 * into *err_word (a device int32; may be NULL).  No out-of-range read occurs.
 * ------------------------------------------------------------------------- */
CBX_API int cbx_embed_gather_add(const void* tok_table, int tok_type, int64_t n_tok_rows,
                                 const void* pos_table, int pos_type, int64_t n_pos_rows,
                                 const int32_t* ids, const int32_t* pos_ids, int64_t pos_offset,
                                 int64_t n_rows, int64_t hidden,
                                 void* out, int out_type,
                                 int32_t* err_word, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Batched prefill gather: n_batch utterances of seq_len tokens each, every
 * utterance at positions n_past .. n_past + seq_len - 1:
 *
 *   out[b][t, :] = tok_table[ids[b][t], :] + pos_table[n_past + t, :]
 *
 * ids: [n_batch][seq_len] int32; out: [n_batch][seq_len][hidden].  The same
 * result as cbx_embed_gather_add over the n_batch * seq_len rows with
 * pos_ids[b * seq_len + t] = n_past + t (the engine's per-utterance gather of
 * chatterbox-cpp/src/t3.cpp:440-455 with the positions of :597-600, for a
 * batch of utterances in one launch), types, rounding and out-of-range
 * handling included.  With one table type, 16-byte aligned rows of at most
 * 256 vectors, the rows are processed position by position so that each
 * position row is read once per warp and reused across the batch.
 * pos_table may be NULL (a plain batched gather).  out must not overlap the
 * inputs.
 * ------------------------------------------------------------------------- */
CBX_API int cbx_embed_gather_add_batched(const void* tok_table, int tok_type, int64_t n_tok_rows,
                                         const void* pos_table, int pos_type, int64_t n_pos_rows,
                                         const int32_t* ids, int64_t n_batch, int64_t seq_len,
                                         int64_t n_past, int64_t hidden, void* out, int out_type,
                                         int32_t* err_word, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * The T3 prefill input sequence in one pass (chatterbox-cpp/src/t3.cpp:428-455,
 * positions filled at :597-600):
 *
 *   seq = [ cond_rows (n_cond rows, f32: the cond_enc GEMM output + bias) ;
 *           prompt_table[prompt_ids]   (the speech table, n_prompt rows)   ;
 *           tok_table[tok_ids]         (text or speech table, n_tok rows)  ]
 *   out[i, :] = seq[i, :] + pos_table[n_past + i, :]
 *
 * i.e. the engine's ggml_get_rows x3, ggml_cast x3, ggml_concat x2 and
 * ggml_add over N = n_cond + n_prompt + n_tok rows.  Rows are widened to f32,
 * added once and rounded once to out_type (the engine's f32: bit-exact).
 * Without a conditioning prefix pass n_cond = n_prompt = 0 (t3.cpp:284, :294).
 * Tables: F32 / F16 / BF16 (the GGUF ships them f16,
 * scripts/convert_chatterbox_to_gguf.py); the fast path wants prompt, token
 * and position tables of one type, 16-byte aligned.  pos_table may be NULL.
 * Out-of-range ids / positions: zero row + CBX_EFLAG_* in *err_word (may be
 * NULL), as cbx_embed_gather_add.  out must not overlap the inputs.
 * ------------------------------------------------------------------------- */
CBX_API int cbx_t3_embed_sequence(const float* cond_rows, int64_t n_cond,
                                  const void* prompt_table, int prompt_type,
                                  int64_t n_prompt_table_rows, const int32_t* prompt_ids,
                                  int64_t n_prompt,
                                  const void* tok_table, int tok_type, int64_t n_tok_table_rows,
                                  const int32_t* tok_ids, int64_t n_tok,
                                  const void* pos_table, int pos_type, int64_t n_pos_rows,
                                  int64_t n_past, int64_t hidden, void* out, int out_type,
                                  int32_t* err_word, cbx_stream_t stream);

/* The same sequence for n_batch utterances in one launch: cond_rows
 * [n_batch][n_cond][hidden] f32, prompt_ids [n_batch][n_prompt], tok_ids
 * [n_batch][n_tok], out [n_batch][N][hidden] with N = n_cond + n_prompt +
 * n_tok; every utterance at positions n_past .. n_past + N - 1.  Utterance b
 * equals cbx_t3_embed_sequence on its own rows, bit for bit.  A server that
 * prefills a batch of requests makes one call instead of n_batch
 * (chatterbox-cpp/src/t3.cpp:428-455 runs one utterance per forward). */
CBX_API int cbx_t3_embed_sequence_batched(const float* cond_rows, int64_t n_cond,
                                          const void* prompt_table, int prompt_type,
                                          int64_t n_prompt_table_rows, const int32_t* prompt_ids,
                                          int64_t n_prompt,
                                          const void* tok_table, int tok_type,
                                          int64_t n_tok_table_rows, const int32_t* tok_ids,
                                          int64_t n_tok,
                                          const void* pos_table, int pos_type, int64_t n_pos_rows,
                                          int64_t n_past, int64_t hidden, int64_t n_batch,
                                          void* out, int out_type, int32_t* err_word,
                                          cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Residual add fused with LayerNorm over ne0 (row-wise).
 *
 *   s = x + resid                      (skipped when resid == NULL: s = x)
 *   y = (s - mean(s)) / sqrt(var(s) + eps) * gamma + beta
 *
 * var is the biased variance.  Statistics are f32-or-better on the f32 value
 * of s (before it is rounded to in_type).  gamma / beta are f32 [hidden]
 * (NULL = 1 / 0).  sum_out (may be NULL) receives s in in_type.
 * in_type ∈ {F32, BF16, F16}; out_type ∈ {F32, BF16, F16}.
 * Strides are in elements between consecutive rows (0 = hidden):
 * in_row_stride for x and resid, out_row_stride for sum_out and y.
 *
 * Replaces chatterbox-cpp/src/t3.cpp:528-532 (ggml_add residual, then
 * ggml_norm + ggml_mul + ggml_add), t3.cpp:541 + :465-466 (residual, next
 * layer's LN1), t3.cpp:545-546 (final LN, resid == NULL), and the layer_norm()
 * helpers at cfm_decoder.cpp:29-33 / flow_encoder.cpp:58-62 (resid == NULL).
 * ------------------------------------------------------------------------- */
CBX_API int cbx_add_layernorm(const void* x, const void* resid, int in_type, int64_t in_row_stride,
                              const float* gamma, const float* beta, float eps,
                              int64_t n_rows, int64_t hidden,
                              void* sum_out, void* y, int out_type, int64_t out_row_stride,
                              cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * CFM CausalBlock1D tail: LayerNorm over the channel axis, activation, mask.
 *
 *   y[b,c,t] = act( LN_c(x[b,:,t]) * gamma[c] + beta[c] ) * mask[b,t]
 *
 * x, y: f32 of B*C*T elements in `layout` (BCT: channel-strided, stride T
 * between channels; BTC: channels contiguous).  mask: f32 [B][T] or NULL
 * (= 1).  act ∈ {NONE, MISH, SILU, GELU_TANH}.
 *
 * Replaces chatterbox-cpp/src/cfm_decoder.cpp:144-148 (layer_norm :29-33,
 * mish :36-38 = ggml_softplus + ggml_tanh + ggml_mul, then ggml_mul by the
 * (1,T) mask); the BCT form is the PyTorch layout of
 * scripts/reference_cfm_decoder.py:241-256 (transpose, LN over C, transpose
 * back, Mish, mask).
 * ------------------------------------------------------------------------- */
CBX_API int cbx_layernorm_channels(const float* x, const float* gamma, const float* beta, float eps,
                                   const float* mask, int64_t B, int64_t C, int64_t T,
                                   int layout, int act, float* y, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * CFM causal conv epilogue + CausalBlock1D tail, one pass:
 *
 *   h[b,c,t] = x[b,c,t] + conv_bias[c]                      (f32, ggml_add)
 *   y[b,t,c] = act( LN_c(h[b,:,t]) * gamma[c] + beta[c] ) * mask[b,t]
 *
 * x: f32 [B][C][T], the causal conv's GEMM output (ggml ne = (T, C_out));
 * y: f32 [B][T][C], the engine's (C, T) activation layout; y must not overlap
 * x.  conv_bias, gamma, beta: f32 [C] or NULL; mask: f32 [B][T] or NULL.
 * act ∈ {NONE, MISH, SILU, GELU_TANH}.
 *
 * Replaces chatterbox-cpp/src/cfm_decoder.cpp:114-115 (add_bias_TC, then
 * ggml_cont(ggml_transpose) back to (C_out, T)) followed by :144-148
 * (layer_norm, mish, ggml_mul by the mask): four passes, here one.
 * ------------------------------------------------------------------------- */
CBX_API int cbx_causal_block1d_tail(const float* x, const float* conv_bias, const float* gamma,
                                    const float* beta, float eps, const float* mask, int64_t B,
                                    int64_t C, int64_t T, int act, float* y,
                                    cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Elementwise activations over n elements, type ∈ {F32, BF16, F16} (compute
 * in f32, one rounding at the store).
 *
 * cbx_gelu_tanh: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
 *   replaces ggml_gelu at chatterbox-cpp/src/t3.cpp:537 (formula of
 *   scripts/reference_t3_forward.py:73-77).
 * cbx_silu: x * sigmoid(x)
 *   replaces ggml_silu at cfm_decoder.cpp:466, flow_encoder.cpp:402
 *   (scripts/reference_cfm_decoder.py:141-142).
 * cbx_mish: x * tanh(softplus(x)), softplus(x) = x for x > 20
 *   replaces mish() at cfm_decoder.cpp:36-38 (used :146, :163;
 *   scripts/reference_cfm_decoder.py:145-149).
 * ------------------------------------------------------------------------- */
CBX_API int cbx_gelu_tanh(const void* x, void* y, int64_t n, int type, cbx_stream_t stream);
CBX_API int cbx_silu(const void* x, void* y, int64_t n, int type, cbx_stream_t stream);
CBX_API int cbx_mish(const void* x, void* y, int64_t n, int type, cbx_stream_t stream);

/* cbx_gelu_erf: exact GELU 0.5 x (1 + erf(x / sqrt 2)); replaces
 * ggml_gelu_erf at chatterbox-cpp/src/cfm_decoder.cpp:239 (transformer FF) and
 * s3enc.cpp:177, :182, :280 (formula of scripts/reference_cfm_decoder.py:152-155). */
CBX_API int cbx_gelu_erf(const void* x, void* y, int64_t n, int type, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * GEMM-epilogue neighbours.
 *
 * cbx_bias_act: y[r, j] = act(x[r, j] + b) over n_rows rows of `hidden`
 * elements (ne0 innermost), the sum rounded to f32 first as ggml_add does.
 * bias may be NULL (plain activation); with bias_axis NE0, b = bias[j]
 * (bias_len must equal hidden); with NE1, b = bias[r % bias_len] (a per-row
 * bias, e.g. C channels of a (T, C) conv output, batch-major rows).
 * act: any cbx_act; act_param is LeakyReLU's slope (ignored otherwise).
 * type ∈ {F32, BF16, F16} for x and y (f32 bias).  Replaces:
 *   chatterbox-cpp/src/t3.cpp:536-537     cur = add(cur, fc_b); gelu(cur)
 *   cfm_decoder.cpp:114 (add_bias_TC)     conv output + per-channel bias
 *   hift_vocoder.cpp:575                  ggml_elu (F0 predictor)
 *   hift_vocoder.cpp:686, :748            ggml_leaky_relu (slopes 0.1, 0.01)
 *
 * cbx_sum3_scale: y = ((a + b) + c) * scale with each ggml node rounded to f32
 * (hift_vocoder.cpp:733-739: the three ResBlocks' sum times 1/3).
 * ------------------------------------------------------------------------- */
CBX_API int cbx_bias_act(const void* x, void* y, int type, int64_t n_rows, int64_t hidden,
                         const float* bias, int bias_axis, int64_t bias_len, int act,
                         float act_param, cbx_stream_t stream);
CBX_API int cbx_sum3_scale(const void* a, const void* b, const void* c, float scale, void* y,
                           int64_t n, int type, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * Sinusoidal timestep embedding (batched), optionally followed by SiLU.
 *
 *   a_ij = (scale * t[i]) * freqs[j]                  (f32, in this order)
 *   y[i, j] = sin(a_ij), y[i, half + j] = cos(a_ij),  j < half = dim / 2
 *   (odd dim: y[i, dim-1] = 0, as the engine's zero-initialised vector)
 *
 * t: device f32 [n_t]; freqs: device f32 [dim/2] built by
 * cbx_sinusoid_freqs; y: device f32 [n_t][dim]; act ∈ {NONE, SILU}.
 * Replaces the host loop sinusoidal_pos_emb() of
 * chatterbox-cpp/src/cfm_decoder.cpp:49-62 (called at :418-419) and the SiLU
 * that follows in the time MLP input path (:466; config: dim 320, scale 1000).
 * ------------------------------------------------------------------------- */
CBX_API int cbx_timestep_embed(const float* t, int64_t n_t, const float* freqs, int32_t dim,
                               float scale, int act, float* y, cbx_stream_t stream);

/* host: freqs[j] = expf(-(logf(10000) / (half - 1)) * j), j < dim/2, with the
 * exact f32 expression of chatterbox-cpp/src/cfm_decoder.cpp:52-56.
 * dim >= 4 (half - 1 must be positive). */
CBX_API int cbx_sinusoid_freqs(int32_t dim, float* freqs_host);

/* ------------------------------------------------------------------------- *
 * HiFT Snake: y = x + sin^2(alpha_c * x) * alpha_inv_c.
 *
 * The composition is ggml's five nodes at chatterbox-cpp/src/hift_vocoder.cpp:
 * 64-73 (mul, sin, sqr, mul, add) fused into one pass.  alpha_inv may be NULL,
 * in which case alpha_inv_c = 1 / (alpha_c + eps) is formed on the device with
 * the f32 expression the engine uses at load (hift_vocoder.cpp:413-427;
 * eps = snake_eps = 1e-9, hift_vocoder.h:72).
 * x, y: f32 of B*C*T elements in `layout`; alpha, alpha_inv: f32 [C].
 * ------------------------------------------------------------------------- */
CBX_API int cbx_snake(const float* x, const float* alpha, const float* alpha_inv, float eps,
                      int64_t B, int64_t C, int64_t T, int layout, float* y,
                      cbx_stream_t stream);

/* host: alpha_inv[c] = 1.0f / (alpha[c] + eps) in f32 (hift_vocoder.cpp:419-420). */
CBX_API int cbx_snake_alpha_inv(const float* alpha_host, int64_t n, float eps, float* alpha_inv_host);

/* ------------------------------------------------------------------------- *
 * T3 attention prologue after the QKV GEMM (chatterbox-cpp/src/t3.cpp:465-489),
 * fused: for each row r (a token),
 *   t = qkv[r][i] + qkv_bias[i]                       (f32, one ggml_add)
 *   q_out[r][i]                       = t,            0 <= i < D   (Q)
 *   cache_k[r*slab_stride + pos*D + i] = (T)t,        D <= i < 2D  (K row)
 *   cache_v[r*slab_stride + pos*D + i] = (T)t,        2D <= i < 3D (V row)
 * with pos = positions[r] (NULL: pos_offset + r) and T = cache_type (the
 * engine's cache is f32, t3.cpp:252-253; f16 / bf16 round to nearest even).
 * A prefill chunk of one stream: positions NULL, pos_offset = n_past,
 * slab_stride 0.  A batched decode step: one row per stream, positions[r] =
 * that stream's n_past, slab_stride = elements between streams' cache slabs.
 * A position outside [0, max_context) writes no cache row and ORs
 * CBX_EFLAG_POS_OOB into *err_word (device int32); q_out may be NULL.  q_out and the
 * caches must not overlap qkv.  With n_rows > 1 a nonzero slab_stride below
 * max_context * D (slabs that overlap) is rejected.  The library sees only
 * pointers: each cache must hold (n_rows - 1) * slab_stride + max_context * D
 * elements, and positions n_rows entries (the Python wrapper checks both).
 * qkv: f32 rows of qkv_row_stride elements (0 = 3D); qkv_bias f32 [3D] or NULL.
 * ------------------------------------------------------------------------- */
CBX_API int cbx_qkv_kv_append(const float* qkv, int64_t qkv_row_stride, const float* qkv_bias,
                              int64_t n_rows, int64_t D, const int32_t* positions,
                              int32_t pos_offset, void* cache_k, void* cache_v, int cache_type,
                              int64_t slab_stride, int64_t max_context, float* q_out,
                              int32_t* err_word, cbx_stream_t stream);

/* ------------------------------------------------------------------------- *
 * HiFT host DSP either side of the Snake stack, on the device.
 *
 * cbx_nsf_source replaces HiFTVocoder::generate_source
 * (chatterbox-cpp/src/hift_vocoder.cpp:853-965) in its explicit form: the
 * caller passes the random phase and noise (the engine's phase_vec_opt /
 * noise_z_opt; phase[b][0] is ignored and taken as 0, as at :885).  Per
 * utterance b and wave sample t = m * upsample + j:
 *   f = f0[b][m]; u = f > 10; noise_amp = u * 0.003f + (1 - u) * (0.1f / 3.0f)
 *   cs_h += (double)f * (h + 1) / sampling_rate      (double, sample order)
 *   sine_h = 0.1f * (float)sin(2 pi frac(cs_h) + phase[b][h])
 *   s = lin_b + sum_h lin_w[h] * (sine_h * u + noise_amp * noise[b][h][t])
 *   out[b][t] = tanhf((float)s)
 * The double running sum is reproduced exactly (closed-form replay of the
 * engine's sequential additions).  f0 f32 [B][n_mel]; phase f32 [B][9];
 * noise f32 [B][9][n_mel * upsample]; lin_w_host: 9 floats in HOST memory (the
 * engine reads l_linear on the host, :948-954); out f32 [B][n_mel * upsample],
 * not overlapping the inputs.  With upsample even and >= 18 and out 8-byte
 * aligned the call runs two kernels, and out holds each frame's running sums
 * between them; it is complete when the call's work on the stream is.
 * ------------------------------------------------------------------------- */
#define CBX_NSF_HARMONICS 9
CBX_API int cbx_nsf_source(const float* f0, int64_t B, int64_t n_mel, int32_t upsample,
                           int32_t sampling_rate, const float* phase, const float* noise,
                           const float* lin_w_host, float lin_b, float* out, cbx_stream_t stream);

/* Centered STFT, stft_centered_host (hift_vocoder.cpp:465-498): reflect padding
 * by n_fft/2, frames every hop samples, frame = x * window (f32), DFT in double,
 * bins rounded to f32.  audio f32 [B][T] (T > n_fft/2); window f32 [n_fft];
 * n_fft even, 2..32; 1 <= hop <= n_fft; T_stft = 1 + T / hop; nb = n_fft/2 + 1.
 * layout BTC: out [B][T_stft][2 nb], each frame's nb real bins then nb imag bins
 * (the engine's s_stft rows, :627-638); BCT: out [B][2 nb][T_stft].  out must not
 * overlap audio. */
CBX_API int cbx_stft(const float* audio, int64_t B, int64_t T, int32_t n_fft, int32_t hop,
                     const float* window, int layout, float* out, cbx_stream_t stream);

/* The HiFT output tail, hift_vocoder.cpp:787-829: from conv_post's 2 nb
 * channels, magnitude = min(expf(raw), 100), phase = sinf(raw), re = mag *
 * cosf(phase), im = mag * sinf(phase) (f32); then istft_centered_host
 * (:501-541): inverse DFT per frame in double, / n_fft, f32 windowed
 * overlap-add in frame order, division by the window-square sum where it is
 * > 1e-11, trim of n_fft/2 per side, clamp to [-audio_limit, audio_limit]
 * (INFINITY: no clamp).  post f32 BTC [B][n_frames][2 nb] (the engine's
 * (T_final, 18) rows) or BCT [B][2 nb][n_frames]; out f32
 * [B][(n_frames - 1) * hop], not overlapping post. */
CBX_API int cbx_istft_post(const float* post, int64_t B, int64_t n_frames, int32_t n_fft,
                           int32_t hop, const float* window, int layout, float audio_limit,
                           float* out, cbx_stream_t stream);

/* host: periodic Hann window, the engine's f32 expression
 * 0.5f - 0.5f * cosf(2.0f * (float)M_PI * n / n_fft) (hift_vocoder.cpp:429-434). */
CBX_API int cbx_hann_window(int32_t n_fft, float* window_host);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* CBX_OPS_H */
