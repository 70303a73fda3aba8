"""CPU oracle for libcbx_ops — TEST INFRASTRUCTURE ONLY.

This package is the checker: tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of bench.py use it to compute the
expected output of every op on the CPU.  The product path
(``chatterbox_amdvulkan_b200``) never imports it.

The arithmetic lives in ``cbx_oracle.c`` (a C restatement of the reference
engine's helper compositions; every function there cites the
chatterbox-cpp/src file:line it follows).  This module only builds it, loads it
with ctypes and exposes NumPy-facing wrappers.  16-bit element types are held
in ``np.uint16`` arrays (raw bf16 / f16 bits); f32 in ``np.float32``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcbx_oracle.so")

F32, F16, BF16 = 0, 1, 30
BCT, BTC = 0, 1
ACT_NONE, ACT_MISH, ACT_SILU, ACT_GELU = 0, 1, 2, 3
ACT_GELU_ERF, ACT_LEAKY_RELU, ACT_ELU = 4, 5, 6
EFLAG_TOKEN_OOB, EFLAG_POS_OOB = 0x1, 0x2   # error-word bits of the gathers
BIAS_NE0, BIAS_NE1 = 0, 1

_lib = None


def build(force: bool = False) -> str:
    """Compile cbx_oracle.c into libcbx_oracle.so with the committed Makefile."""
    src = os.path.join(HERE, "cbx_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "-B", "libcbx_oracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        sig = {
            "cbxo_embed_gather_add": [vp, i32, i64, vp, i32, i64, vp, vp, i64, i64, i64, vp, i32, vp],
            "cbxo_add_layernorm_act": [vp, vp, i32, i64, vp, vp, f32, i64, i64, vp, vp, i32, i64,
                                       i32, vp],
            "cbxo_add_layernorm": [vp, vp, i32, i64, vp, vp, f32, i64, i64, vp, vp, i32, i64],
            "cbxo_layernorm_channels": [vp, vp, vp, f32, vp, i64, i64, i64, i32, i32, vp],
            "cbxo_gelu_tanh": [vp, vp, i64, i32],
            "cbxo_gelu_erf": [vp, vp, i64, i32],
            "cbxo_bias_act": [vp, vp, i32, i64, i64, vp, i32, i64, i32, f32],
            "cbxo_sum3_scale": [vp, vp, vp, f32, vp, i64, i32],
            "cbxo_silu": [vp, vp, i64, i32],
            "cbxo_mish": [vp, vp, i64, i32],
            "cbxo_sinusoid_freqs": [i32, vp],
            "cbxo_timestep_embed": [vp, i64, vp, i32, f32, i32, vp],
            "cbxo_snake_alpha_inv": [vp, i64, f32, vp],
            "cbxo_snake": [vp, vp, vp, f32, i64, i64, i64, i32, vp],
            "cbxo_nsf_source": [vp, i64, i64, i32, i32, vp, vp, vp, f32, vp],
            "cbxo_qkv_kv_append": [vp, i64, vp, i64, i64, vp, i32, vp, vp, i32, i64, i64, vp, vp],
            "cbxo_hann_window": [i32, vp],
            "cbxo_stft": [vp, i64, i64, i32, i32, vp, i32, vp],
            "cbxo_istft_post": [vp, i64, i64, i32, i32, vp, i32, f32, vp],
            "cbxo_set_threads": [i32],
            "cbxo_max_threads": [],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        for name in ("cbxo_f32_to_type", "cbxo_type_to_f32"):
            fn = getattr(L, name)
            fn.argtypes = [vp, vp, i64, i32]
            fn.restype = None
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _check(rc, name):
    if rc != 0:
        raise ValueError(f"{name} rejected its arguments (status {rc})")


def set_threads(n: int) -> int:
    return lib().cbxo_set_threads(int(n))


def max_threads() -> int:
    return lib().cbxo_max_threads()


def storage_dtype(t: int):
    return np.float32 if t == F32 else np.uint16


# ----------------------------------------------------------------- dtypes --

def to_type(x_f32: np.ndarray, t: int) -> np.ndarray:
    """Round an f32 array to element type t (RNE); returns its storage array."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    if t == F32:
        return x.copy()
    out = np.empty(x.shape, np.uint16)
    lib().cbxo_f32_to_type(_p(x), _p(out), x.size, t)
    return out


def to_f32(a: np.ndarray, t: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if t == F32:
        return a.astype(np.float32, copy=True)
    out = np.empty(a.shape, np.float32)
    lib().cbxo_type_to_f32(_p(a), _p(out), a.size, t)
    return out


# -------------------------------------------------------------------- ops --

def embed_gather_add(tok, tok_t, ids, pos=None, pos_t=F32, pos_ids=None, pos_offset=0,
                     out_t=F32):
    """out[i] = tok[ids[i]] + pos[p_i] (t3.cpp:440-455).  Returns (out, err_bits)."""
    ids = np.ascontiguousarray(ids, np.int32)
    n_rows = ids.shape[0]
    hidden = tok.shape[1]
    out = np.empty((n_rows, hidden), storage_dtype(out_t))
    err = np.zeros(1, np.int32)
    pid = None if pos_ids is None else np.ascontiguousarray(pos_ids, np.int32)
    rc = lib().cbxo_embed_gather_add(_p(np.ascontiguousarray(tok)), tok_t, tok.shape[0],
                                     _p(None if pos is None else np.ascontiguousarray(pos)),
                                     pos_t, 0 if pos is None else pos.shape[0],
                                     _p(ids), _p(pid), int(pos_offset), n_rows, hidden,
                                     _p(out), out_t, _p(err))
    _check(rc, "embed_gather_add")
    return out, int(err[0])


def t3_embed_sequence(tok, tok_t, tok_ids, pos=None, pos_t=F32, n_past=0, cond=None,
                      prompt=None, prompt_t=F32, prompt_ids=None, out_t=F32):
    """The T3 prefill input sequence, node by node as chatterbox-cpp builds it
    (t3.cpp:428-455): seq = concat(cond_emb, cast_f32(get_rows(speech_emb,
    prompt)), cast_f32(get_rows(emb_table, tokens))) along the rows, then
    h = seq + cast_f32(get_rows(pos_embd, n_past + i)), one f32 add, rounded to
    out_t.  An out-of-range id or position gives a zero row and its flag bit
    (the kernel's contract; the engine itself does not check).
    Returns (out, err_bits)."""
    H = tok.shape[1]
    parts, flags = [], 0

    def gathered(table, t, ids):
        nonlocal flags
        ids = np.asarray(ids, np.int64)
        bad = (ids < 0) | (ids >= table.shape[0])
        flags |= EFLAG_TOKEN_OOB if bad.any() else 0
        rows = to_f32(table[np.where(bad, 0, ids)], t)
        rows[bad] = 0.0
        return rows, bad

    bad_rows = []
    if cond is not None:
        c = np.asarray(cond, np.float32).reshape(-1, H)
        parts.append(c.copy())
        bad_rows.append(np.zeros(c.shape[0], bool))
    if prompt_ids is not None and len(prompt_ids):
        r, b = gathered(prompt, prompt_t, prompt_ids)
        parts.append(r)
        bad_rows.append(b)
    r, b = gathered(tok, tok_t, tok_ids)
    parts.append(r)
    bad_rows.append(b)
    seq = np.concatenate(parts, axis=0) if parts else np.zeros((0, H), np.float32)
    bad = np.concatenate(bad_rows) if bad_rows else np.zeros(0, bool)
    n = seq.shape[0]
    if pos is not None:
        p = n_past + np.arange(n, dtype=np.int64)
        pbad = (p < 0) | (p >= pos.shape[0])
        flags |= EFLAG_POS_OOB if pbad.any() else 0
        prow = to_f32(pos[np.where(pbad, 0, p)], pos_t)
        seq = (seq + prow).astype(np.float32)        # ggml_add in f32
        bad = bad | pbad
    seq[bad] = 0.0
    return to_type(seq, out_t), flags


def add_layernorm(x, resid, gamma, beta, eps, in_t=F32, out_t=F32, act=ACT_NONE, mask=None):
    """(s, y) of residual-add + LayerNorm over the last axis (t3.cpp:528-532)."""
    x = np.ascontiguousarray(x)
    H = x.shape[-1]
    n_rows = x.size // H
    r = None if resid is None else np.ascontiguousarray(resid)
    s = np.empty(x.shape, storage_dtype(in_t))
    y = np.empty(x.shape, storage_dtype(out_t))
    g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
    b = None if beta is None else np.ascontiguousarray(beta, np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, np.float32)
    rc = lib().cbxo_add_layernorm_act(_p(x), _p(r), in_t, H, _p(g), _p(b), float(eps), n_rows,
                                      H, _p(s), _p(y), out_t, H, act, _p(m))
    _check(rc, "add_layernorm")
    return s, y


def layernorm_channels(x, gamma, beta, eps, mask=None, layout=BCT, act=ACT_MISH):
    """CausalBlock1D tail (cfm_decoder.cpp:144-148) on f32 x of shape [B,C,T] or [B,T,C]."""
    x = np.ascontiguousarray(x, np.float32)
    if layout == BCT:
        B, C, T = x.shape
    else:
        B, T, C = x.shape
    y = np.empty_like(x)
    m = None if mask is None else np.ascontiguousarray(mask, np.float32)
    g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
    b = None if beta is None else np.ascontiguousarray(beta, np.float32)
    rc = lib().cbxo_layernorm_channels(_p(x), _p(g), _p(b), float(eps), _p(m), B, C, T, layout,
                                       act, _p(y))
    _check(rc, "layernorm_channels")
    return y


def causal_block1d_tail(x, conv_bias, gamma, beta, eps, mask=None, act=ACT_MISH):
    """The causal conv's epilogue and the CausalBlock1D tail
    (cfm_decoder.cpp:114-115, :144-148): h = x + conv_bias[c] (ggml_add, f32),
    transposed from the GEMM's [B,C,T] to the engine's [B,T,C]
    (ggml_cont(ggml_transpose)), then LN over C, act and mask.  x: f32
    [B,C,T]; returns f32 [B,T,C]."""
    x = np.ascontiguousarray(x, np.float32)
    h = x if conv_bias is None else (x + np.asarray(conv_bias, np.float32)[None, :, None])
    h = np.ascontiguousarray(h.astype(np.float32).transpose(0, 2, 1))
    return layernorm_channels(h, gamma, beta, eps, mask, BTC, act)


def _unary(name, x, t):
    x = np.ascontiguousarray(x)
    y = np.empty_like(x)
    _check(getattr(lib(), name)(_p(x), _p(y), x.size, t), name)
    return y


def gelu_tanh(x, t=F32):
    return _unary("cbxo_gelu_tanh", x, t)


def gelu_erf(x, t=F32):
    return _unary("cbxo_gelu_erf", x, t)


def bias_act(x, bias=None, axis=BIAS_NE0, act=ACT_NONE, param=0.0, t=F32, bias_len=None):
    """act(x + bias) over rows of x.shape[-1] elements (t3.cpp:536-537 and neighbours)."""
    x = np.ascontiguousarray(x)
    H = x.shape[-1]
    n_rows = x.size // H
    y = np.empty_like(x)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    blen = (b.size if b is not None else 0) if bias_len is None else bias_len
    _check(lib().cbxo_bias_act(_p(x), _p(y), t, n_rows, H, _p(b), axis, blen, act,
                               float(param)), "bias_act")
    return y


def sum3_scale(a, b, c, scale, t=F32):
    """((a + b) + c) * scale with f32 node rounding (hift_vocoder.cpp:733-739)."""
    a, b, c = (np.ascontiguousarray(v) for v in (a, b, c))
    y = np.empty_like(a)
    _check(lib().cbxo_sum3_scale(_p(a), _p(b), _p(c), float(scale), _p(y), a.size, t),
           "sum3_scale")
    return y


def silu(x, t=F32):
    return _unary("cbxo_silu", x, t)


def mish(x, t=F32):
    return _unary("cbxo_mish", x, t)


def sinusoid_freqs(dim: int) -> np.ndarray:
    out = np.empty(dim // 2, np.float32)
    _check(lib().cbxo_sinusoid_freqs(int(dim), _p(out)), "sinusoid_freqs")
    return out


def timestep_embed(t, dim, scale=1000.0, act=ACT_NONE, freqs=None):
    t = np.ascontiguousarray(t, np.float32).reshape(-1)
    fr = sinusoid_freqs(dim) if freqs is None else np.ascontiguousarray(freqs, np.float32)
    y = np.empty((t.shape[0], dim), np.float32)
    _check(lib().cbxo_timestep_embed(_p(t), t.shape[0], _p(fr), int(dim), float(scale), act,
                                     _p(y)), "timestep_embed")
    return y


def snake_alpha_inv(alpha, eps=1e-9):
    a = np.ascontiguousarray(alpha, np.float32)
    inv = np.empty_like(a)
    _check(lib().cbxo_snake_alpha_inv(_p(a), a.size, float(eps), _p(inv)), "snake_alpha_inv")
    return inv


def snake(x, alpha, alpha_inv=None, eps=1e-9, layout=BCT):
    """Snake on f32 x of shape [B,C,T] (BCT) or [B,T,C] (BTC) (hift_vocoder.cpp:64-73)."""
    x = np.ascontiguousarray(x, np.float32)
    if layout == BCT:
        B, C, T = x.shape
    else:
        B, T, C = x.shape
    y = np.empty_like(x)
    a = np.ascontiguousarray(alpha, np.float32)
    ai = None if alpha_inv is None else np.ascontiguousarray(alpha_inv, np.float32)
    _check(lib().cbxo_snake(_p(x), _p(a), _p(ai), float(eps), B, C, T, layout, _p(y)), "snake")
    return y


NSF_HARM = 9


def nsf_source(f0, upsample, phase, noise, lin_w, lin_b=0.0, sampling_rate=24000):
    """HiFT NSF source (hift_vocoder.cpp:853-965) from f0 [B, n_mel], phase
    [B, 9], noise [B, 9, n_mel*upsample]; returns [B, n_mel*upsample] f32."""
    f0 = np.ascontiguousarray(f0, np.float32)
    if f0.ndim == 1:
        f0 = f0[None]
    B, n_mel = f0.shape
    T = n_mel * int(upsample)
    ph = np.ascontiguousarray(phase, np.float32).reshape(B, NSF_HARM)
    nz = np.ascontiguousarray(noise, np.float32).reshape(B, NSF_HARM, T)
    w = np.ascontiguousarray(lin_w, np.float32).reshape(NSF_HARM)
    out = np.empty((B, T), np.float32)
    _check(lib().cbxo_nsf_source(_p(f0), B, n_mel, int(upsample), int(sampling_rate), _p(ph),
                                 _p(nz), _p(w), float(lin_b), _p(out)), "nsf_source")
    return out


def hann_window(n_fft=16):
    w = np.empty(n_fft, np.float32)
    _check(lib().cbxo_hann_window(n_fft, _p(w)), "hann_window")
    return w


def stft(audio, n_fft=16, hop=4, window=None, layout=BTC):
    """Centered STFT (hift_vocoder.cpp:465-498) of f32 audio [B, T]: BTC ->
    [B, T_stft, 2*nb] (real bins then imag bins per frame), BCT -> [B, 2*nb, T_stft]."""
    x = np.ascontiguousarray(audio, np.float32)
    if x.ndim == 1:
        x = x[None]
    B, T = x.shape
    w = hann_window(n_fft) if window is None else np.ascontiguousarray(window, np.float32)
    nb = n_fft // 2 + 1
    Ts = 1 + (T + 2 * (n_fft // 2) - n_fft) // hop
    out = np.empty((B, Ts, 2 * nb) if layout == BTC else (B, 2 * nb, Ts), np.float32)
    _check(lib().cbxo_stft(_p(x), B, T, n_fft, hop, _p(w), layout, _p(out)), "stft")
    return out


def istft_post(post, n_fft=16, hop=4, window=None, layout=BTC, audio_limit=0.99):
    """HiFT output tail (hift_vocoder.cpp:787-829): conv_post channels ->
    magnitude/phase -> centered iSTFT -> clamp.  post BTC [B, T_f, 2*nb] or BCT
    [B, 2*nb, T_f]; returns [B, (T_f - 1)*hop] f32."""
    x = np.ascontiguousarray(post, np.float32)
    if x.ndim == 2:
        x = x[None]
    B = x.shape[0]
    Tf = x.shape[1] if layout == BTC else x.shape[2]
    w = hann_window(n_fft) if window is None else np.ascontiguousarray(window, np.float32)
    out = np.empty((B, (Tf - 1) * hop), np.float32)
    _check(lib().cbxo_istft_post(_p(x), B, Tf, n_fft, hop, _p(w), layout, float(audio_limit),
                                 _p(out)), "istft_post")
    return out


def qkv_kv_append(qkv, bias, cache_k, cache_v, cache_t=F32, positions=None, pos_offset=0,
                  slab_stride=0, max_context=None, with_q=True):
    """T3 QKV epilogue (t3.cpp:465-489): returns (q [n_rows, D] f32 or None,
    err bits); cache_k / cache_v (oracle storage arrays) are updated in place."""
    x = np.ascontiguousarray(qkv, np.float32)
    n_rows, D3 = x.shape
    D = D3 // 3
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    pos = None if positions is None else np.ascontiguousarray(positions, np.int32)
    if max_context is None:
        raise ValueError("max_context required")
    q = np.empty((n_rows, D), np.float32) if with_q else None
    err = np.zeros(1, np.int32)
    _check(lib().cbxo_qkv_kv_append(_p(x), D3, _p(b), n_rows, D, _p(pos), int(pos_offset),
                                    _p(cache_k), _p(cache_v), cache_t, int(slab_stride),
                                    int(max_context), _p(q), _p(err)), "qkv_kv_append")
    return q, int(err[0])
