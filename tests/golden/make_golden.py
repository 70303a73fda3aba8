"""Generate tests/golden/ref_ops.npz from the reference's own NumPy oracles.

The reference project (tarekedOz/Chatterbox_AMDVulkan) ships per-component
fp32 NumPy re-implementations under scripts/reference_*.py; their op-level
helpers are exactly the formulas the engine's ggml compositions follow:

  reference_t3_forward.py:73-77      gelu_new (GELU-tanh)
  reference_t3_forward.py:80-84      layer_norm (biased variance)
  reference_t3_forward.py:163-170    text_emb[ids] + wpe[:L]  (embedding add)
  reference_cfm_decoder.py:141-142   silu
  reference_cfm_decoder.py:145-149   mish (softplus threshold 20)
  reference_cfm_decoder.py:173-179   layer_norm (LN_EPS = 1e-5)
  reference_cfm_decoder.py:217-224   sinusoidal_pos_emb
  reference_cfm_decoder.py:241-256   LN over C of a [B,C,T] tensor, Mish, mask
  reference_hift_vocoder.py:140-145  snake
  reference_cfm_decoder.py:152-155   gelu (exact, erf)
  reference_hift_vocoder.py:132-137  elu, leaky_relu
  reference_t3_forward.py:126-131    ffn_block: gelu_new(x @ up_w + up_b)
  reference_hift_vocoder.py:446-448  ResBlock average xs / 3
  reference_hift_vocoder.py:243-290  nearest_upsample + nsf_source (SineGen + HnNSF)
  reference_hift_vocoder.py:294-348  hann_window, stft_centered, istft_centered
  reference_hift_vocoder.py:455-465  magnitude / phase -> iSTFT -> clip (decode tail)
  reference_t3_forward.py:105-108    qkv = x @ w + b, then the q / k / v column split
  reference_cfm_decoder.py:199-202, :238-251  conv bias, LN over C, Mish, mask

  reference_t3_forward.py:150-172    the prefill sequence [cond ; speech[prompt] ;
                                     text[ids]] + wpe, caught at the first layer_norm

This script imports those functions from a checkout of the reference (given
by --reference-root or $CBX_REFERENCE_ROOT), runs them on small seeded inputs and
writes inputs and outputs to ref_ops.npz next to this file.  It runs only
where the reference checkout exists; the tests read the committed .npz.

    python tests/golden/make_golden.py --reference-root DIR
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    scripts = os.path.join(root, "scripts")
    if not os.path.isdir(scripts):
        raise SystemExit(f"reference scripts not found under {scripts}")
    sys.path.insert(0, scripts)
    t3 = importlib.import_module("reference_t3_forward")
    cfm = importlib.import_module("reference_cfm_decoder")
    hift = importlib.import_module("reference_hift_vocoder")
    return t3, cfm, hift


def _with_edges(x: np.ndarray, rng) -> np.ndarray:
    """Plant the edge values the ops must handle: ±20 outliers, zeros, tiny and
    moderately large magnitudes."""
    flat = x.reshape(-1)
    edges = np.array([0.0, -0.0, 1e-7, -1e-7, 1e-3, -1e-3, 0.5, -0.5, 3.0, -3.0, 5.0, -5.0,
                      9.5, -9.5, 15.0, -15.0, 19.99, 20.0, 20.01, -20.0, 25.0, -25.0, 40.0,
                      -40.0], np.float32)
    flat[: edges.size] = edges
    idx = rng.choice(flat.size, size=max(1, flat.size // 100), replace=False)
    flat[idx] = np.where(rng.random(idx.size) < 0.5, -20.0, 20.0).astype(np.float32)
    return x


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=os.environ.get("CBX_REFERENCE_ROOT"),
                    help="checkout of the reference project (or $CBX_REFERENCE_ROOT)")
    ap.add_argument("--out", default=os.path.join(HERE, "ref_ops.npz"))
    args = ap.parse_args()
    if not args.reference_root:
        ap.error("give --reference-root or set CBX_REFERENCE_ROOT")
    t3, cfm, hift = _import_reference(args.reference_root)

    rng = np.random.default_rng(20251201)
    g = {}

    # --- GELU-tanh (T3 FFN) ---------------------------------------------------
    x = _with_edges(rng.standard_normal((48, 256)).astype(np.float32) * 3.0, rng)
    g["gelu_x"] = x
    g["gelu_y"] = t3.gelu_new(x).astype(np.float32)

    # --- residual add + LayerNorm (T3, hidden 1024, eps 1e-5) ----------------
    x = _with_edges(rng.standard_normal((24, 1024)).astype(np.float32), rng)
    r = rng.standard_normal((24, 1024)).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    s = (x + r).astype(np.float32)          # h = h + attention_block(...)
    g["ln_x"], g["ln_r"], g["ln_w"], g["ln_b"] = x, r, w, b
    g["ln_s"] = s
    g["ln_y"] = t3.layer_norm(s, w, b, t3.LN_EPS).astype(np.float32)
    # ragged hidden (not a multiple of the vector width)
    x2 = rng.standard_normal((7, 333)).astype(np.float32) * 2.0 + 0.5
    w2 = (1.0 + 0.1 * rng.standard_normal(333)).astype(np.float32)
    b2 = (0.1 * rng.standard_normal(333)).astype(np.float32)
    g["ln2_x"], g["ln2_w"], g["ln2_b"] = x2, w2, b2
    g["ln2_y"] = t3.layer_norm(x2, w2, b2, t3.LN_EPS).astype(np.float32)

    # --- SiLU / Mish (CFM) ---------------------------------------------------
    x = _with_edges(rng.standard_normal((32, 320)).astype(np.float32) * 4.0, rng)
    g["act_x"] = x
    g["silu_y"] = cfm.silu(x)
    g["mish_y"] = cfm.mish(x)

    # --- CFM CausalBlock1D tail: LN over C (+Mish, mask) in [B,C,T] ----------
    B, C, T = 2, 256, 37
    h = rng.standard_normal((B, C, T)).astype(np.float32)
    h[0, :, 3] *= 20.0                        # a column with large values
    lw = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    lb = (0.1 * rng.standard_normal(C)).astype(np.float32)
    mask = np.ones((B, 1, T), np.float32)
    mask[1, 0, T - 5:] = 0.0                  # padded tail of the second item
    # reference_cfm_decoder.py:249-256, without the conv that precedes it.
    h_tc = cfm.layer_norm(h.transpose(0, 2, 1), lw, lb)
    y = cfm.mish(h_tc.transpose(0, 2, 1))
    g["cfm_x"], g["cfm_w"], g["cfm_b"], g["cfm_mask"] = h, lw, lb, mask.reshape(B, T)
    g["cfm_y"] = (y * mask).astype(np.float32)
    g["cfm_ln_only"] = h_tc.transpose(0, 2, 1).astype(np.float32)

    # --- sinusoidal timestep embedding (dim 320, scale 1000) -----------------
    ts = np.concatenate([np.array([0.0, 1.0, 0.5, 1e-3], np.float32),
                         rng.random(12).astype(np.float32)])
    g["sin_t"] = ts
    g["sin_y"] = np.concatenate([cfm.sinusoidal_pos_emb(float(t), 320, 1000.0) for t in ts])
    g["sin_y_scale1"] = np.concatenate([cfm.sinusoidal_pos_emb(float(t), 320, 1.0) for t in ts])
    g["sin_silu_y"] = cfm.silu(g["sin_y"])

    # --- HiFT Snake ([1,C,T], alpha = exp(N(0,0.3))) -------------------------
    C, T = 64, 101
    alpha = np.exp(0.3 * rng.standard_normal(C)).astype(np.float32)
    xs = _with_edges(rng.standard_normal((1, C, T)).astype(np.float32), rng)
    g["snake_x"], g["snake_alpha"] = xs, alpha
    g["snake_y"] = hift.snake(xs, alpha)

    # --- embedding gather-add (T3: text_emb[ids] + wpe[n_past : n_past+L]) ----
    V, P, H = 97, 50, 64
    tok32 = (0.02 * rng.standard_normal((V, H))).astype(np.float32)
    pos32 = (0.02 * rng.standard_normal((P, H))).astype(np.float32)
    ids = rng.integers(0, V, size=19).astype(np.int32)
    ids[0], ids[-1] = 0, V - 1                # table edges
    n_past = 7
    g["emb_tok"], g["emb_pos"], g["emb_ids"] = tok32, pos32, ids
    g["emb_npast"] = np.array([n_past], np.int32)
    g["emb_y"] = (tok32[ids] + pos32[n_past:n_past + ids.size]).astype(np.float32)
    # f16 tables, as the shipped GGUF stores 2-D tensors
    # (convert_chatterbox_to_gguf.py:286-287); the engine casts to f32 then adds.
    tok16, pos16 = tok32.astype(np.float16), pos32.astype(np.float16)
    g["emb_tok16"], g["emb_pos16"] = tok16.view(np.uint16), pos16.view(np.uint16)
    g["emb16_y"] = (tok16.astype(np.float32)[ids]
                    + pos16.astype(np.float32)[n_past:n_past + ids.size]).astype(np.float32)

    # --- GEMM-epilogue neighbours ----------------------------------------------
    # exact GELU (CFM transformer FF, reference_cfm_decoder.py:152-155)
    x = _with_edges(rng.standard_normal((16, 256)).astype(np.float32) * 3.0, rng)
    g["gerf_x"], g["gerf_y"] = x, cfm.gelu(x)
    # ELU and LeakyReLU (HiFT, reference_hift_vocoder.py:132-137)
    g["elu_y"] = hift.elu(x)
    g["lrelu01_y"] = hift.leaky_relu(x, 0.1)
    g["lrelu001_y"] = hift.leaky_relu(x, 0.01)
    # T3 FFN: h = x @ up_w + up_b; gelu_new(h)  (reference_t3_forward.py:126-131)
    hb = rng.standard_normal((12, 512)).astype(np.float32)
    fb = (0.5 * rng.standard_normal(512)).astype(np.float32)
    g["fc_h"], g["fc_b"] = hb, fb
    g["fc_y"] = t3.gelu_new((hb + fb).astype(np.float32)).astype(np.float32)
    # conv bias on (C, T) rows: out + b.reshape(-1, 1) (reference_cfm_decoder.py:200-202)
    cx = rng.standard_normal((80, 37)).astype(np.float32)
    cb = rng.standard_normal(80).astype(np.float32)
    g["cb_x"], g["cb_b"] = cx, cb
    g["cb_y"] = (cx + cb.reshape(-1, 1)).astype(np.float32)
    # HiFT ResBlock average: xs = sum of three ResBlock outputs, x = xs / 3
    # (reference_hift_vocoder.py:446-448)
    r3 = [rng.standard_normal((64, 101)).astype(np.float32) for _ in range(3)]
    g["rb_r0"], g["rb_r1"], g["rb_r2"] = r3
    g["rb_y"] = (sum(r3) / 3.0).astype(np.float32)

    # --- HiFT source and STFT / iSTFT ------------------------------------------
    # NSF source.  The NumPy oracle sums the per-sample phase increments in f32
    # (np.cumsum), the engine in double (hift_vocoder.cpp:925-934); f0 values
    # whose increments f0*(h+1)/24000 are short dyadic fractions make both sums
    # exact, so the fixture pins the formula rather than f32 rounding drift.
    # 5.859375 Hz is unvoiced (<= 10 Hz); 0 Hz is silence.
    f0 = np.array([0.0, 187.5, 93.75, 375.0, 5.859375, 281.25, 11.71875, 187.5], np.float32)
    up = 480
    lw = (0.5 * rng.standard_normal((1, 9))).astype(np.float32)
    lb = np.array([0.05], np.float32)
    state = {"mel2wav.m_source.l_linear.weight": lw, "mel2wav.m_source.l_linear.bias": lb}
    src, phase, noise = hift.nsf_source(hift.nearest_upsample(f0[None], up), state, seed=11,
                                        return_rng_inputs=True)
    g["nsf_f0"], g["nsf_lw"], g["nsf_lb"] = f0, lw.reshape(9), lb
    g["nsf_phase"], g["nsf_noise"] = phase.reshape(1, 9), noise.reshape(1, 9, -1)
    g["nsf_y"] = src.reshape(1, -1).astype(np.float32)
    # periodic Hann (n_fft 16) and the centered STFT of a [2, 203] signal
    win = hift.hann_window(16)
    g["hann16"] = win
    audio = (0.3 * rng.standard_normal((2, 203))).astype(np.float32)
    re, im = hift.stft_centered(audio, 16, 4, win)
    g["stft_x"], g["stft_y"] = audio, np.concatenate([re, im], axis=1).astype(np.float32)
    # decode tail: conv_post channels (18, T_final) -> magnitude (clipped at 100)
    # and phase -> iSTFT -> clip to +-0.99
    Tf = 64
    post = np.concatenate([rng.normal(-2.0, 0.8, (9, Tf)), rng.normal(0.0, 2.0, (9, Tf))])
    post = post.astype(np.float32)
    post[0, 5], post[3, 7] = 5.0, 6.0          # exp > 100: the magnitude clamp
    mag = np.clip(np.exp(post[:9]), None, 1e2)
    phs = np.sin(post[9:])
    wav = hift.istft_centered((mag * np.cos(phs))[None], (mag * np.sin(phs))[None], 16, 4, win)
    g["istft_post"] = post
    g["istft_y"] = np.clip(wav, -hift.AUDIO_LIMIT, hift.AUDIO_LIMIT).astype(np.float32)

    # --- T3 QKV epilogue: qkv = x @ w + b, q / k / v = column thirds ------------
    # attention_block (reference_t3_forward.py:93-120) has no entry point for
    # its first lines, so they are restated here verbatim in meaning: the bias
    # add on the GEMM output and the [0, D), [D, 2D), [2D, 3D) split.
    D = 64
    h = rng.standard_normal((5, 3 * D)).astype(np.float32)
    qb = (0.1 * rng.standard_normal(3 * D)).astype(np.float32)
    qkv = (h + qb).astype(np.float32)
    g["kv_h"], g["kv_b"] = h, qb
    g["kv_q"], g["kv_k"], g["kv_v"] = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]

    # --- CFM causal conv epilogue: bias, LN over C, Mish, mask -----------------
    # causal_block1d (reference_cfm_decoder.py:238-251) after the conv's GEMM:
    # conv1d adds the bias as out + b.reshape(-1, 1) (:199-202), then LN over C,
    # Mish and the mask.  The engine's tensor is (C, T) in ggml order, i.e.
    # [T][C] in memory, so the fixture's output is the [B][T][C] transpose.
    B, C, T = 2, 256, 44
    xc = (2.0 * rng.standard_normal((B, C, T))).astype(np.float32)
    xc[1, :, 7] *= 15.0                       # a column with large values
    cb = (0.5 * rng.standard_normal(C)).astype(np.float32)
    lw = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    lb = (0.1 * rng.standard_normal(C)).astype(np.float32)
    mask = np.ones((B, 1, T), np.float32)
    mask[0, 0, T - 9:] = 0.0
    h = (xc + cb.reshape(-1, 1)).astype(np.float32)
    h_tc = cfm.layer_norm(h.transpose(0, 2, 1), lw, lb)
    y = (cfm.mish(h_tc.transpose(0, 2, 1)) * mask).astype(np.float32)
    g["cbt_x"], g["cbt_cb"], g["cbt_w"], g["cbt_b"] = xc, cb, lw, lb
    g["cbt_mask"] = mask.reshape(B, T)
    g["cbt_y"] = np.ascontiguousarray(y.transpose(0, 2, 1))

    # --- the T3 prefill input sequence, taken from t3_forward itself ---------
    # reference_t3_forward.py:150-172 builds h = concat([cond_spkr, speech_emb
    # [prompt], text_emb[text]]) + wpe[:L] and hands it to the first
    # layer_norm; the fixture catches that argument (a stand-in layer_norm
    # records it and stops the forward) from a small random state.  Tables
    # hold f16-representable values, so the f16 tables of the GGUF give the
    # same sums.
    srng = np.random.default_rng(20261202)
    H, n_sp, n_tx, P = 64, 40, 90, 200

    def f16vals(shape, std):
        return (std * srng.standard_normal(shape)).astype(np.float16).astype(np.float32)

    state = {"cond_enc.spkr_enc.weight": (0.1 * srng.standard_normal((H, 256))).astype(np.float32),
             "cond_enc.spkr_enc.bias": (0.1 * srng.standard_normal(H)).astype(np.float32),
             "speech_emb.weight": f16vals((n_sp, H), 0.02),
             "text_emb.weight": f16vals((n_tx, H), 0.02),
             "tfmr.wpe.weight": f16vals((P, H), 0.02),
             # read as the first layer_norm's arguments (never applied)
             "tfmr.h.0.ln_1.weight": np.ones(H, np.float32),
             "tfmr.h.0.ln_1.bias": np.zeros(H, np.float32)}
    spk = srng.standard_normal(256).astype(np.float32)
    prompt = [int(v) for v in srng.integers(0, n_sp, 23)]
    text = [int(v) for v in srng.integers(0, n_tx, 31)]
    caught = {}

    class _Stop(Exception):
        pass

    def first_layer_norm(x, *args, **kw):
        caught["h"] = np.array(x, dtype=np.float32, copy=True)
        raise _Stop

    real_ln = t3.layer_norm
    t3.layer_norm = first_layer_norm
    try:
        t3.t3_forward(state, spk, prompt, text)
    except _Stop:
        pass
    finally:
        t3.layer_norm = real_ln
    g["seq_cond"] = (spk @ state["cond_enc.spkr_enc.weight"].T
                     + state["cond_enc.spkr_enc.bias"]).astype(np.float32)
    g["seq_speech16"] = state["speech_emb.weight"].astype(np.float16).view(np.uint16)
    g["seq_text16"] = state["text_emb.weight"].astype(np.float16).view(np.uint16)
    g["seq_pos16"] = state["tfmr.wpe.weight"].astype(np.float16).view(np.uint16)
    g["seq_prompt_ids"] = np.array(prompt, np.int32)
    g["seq_text_ids"] = np.array(text, np.int32)
    g["seq_y"] = caught["h"]

    np.savez_compressed(args.out, **g)
    print(f"wrote {args.out}: {len(g)} arrays, {os.path.getsize(args.out)} bytes")


if __name__ == "__main__":
    main()
