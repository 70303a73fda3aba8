"""Torch-facing wrappers of libcbx_ops, named after the engine's layer helpers.

Each function takes CUDA tensors (the device memory), enqueues one kernel of
libcbx_ops on the current torch CUDA stream through the C ABI, and returns the
output tensor.  The names and argument meanings follow the chatterbox-cpp
helpers they replace:

  embed_gather_add   t3.cpp:432-455      get_rows x2 + cast + concat + add
  t3_embed_sequence  t3.cpp:428-455      [cond ; speech[prompt] ; tokens] + pos
  add_layernorm      t3.cpp:528-532      residual add, norm, mul(w), add(b)
  layer_norm         cfm_decoder.cpp:29  layer_norm(ctx, x, w, b, eps)
  layernorm_channels cfm_decoder.cpp:144-148  LN over C, mish, * mask
  gelu / silu / mish t3.cpp:537, cfm_decoder.cpp:466, cfm_decoder.cpp:36
  gelu_erf           cfm_decoder.cpp:239, s3enc.cpp:177
  bias_act           t3.cpp:536-537 (fc bias + GELU), cfm_decoder.cpp:114,
                     hift_vocoder.cpp:575 (ELU), :686 / :748 (LeakyReLU)
  sum3_scale         hift_vocoder.cpp:733-739 (ResBlock average)
  sinusoidal_pos_emb cfm_decoder.cpp:49-62 (batched, on the device)
  snake              hift_vocoder.cpp:64-73

There is no CPU path: inputs must be CUDA tensors and the shared library must
be present, otherwise these raise.
"""
from __future__ import annotations

import ctypes
import functools

import numpy as np
import torch

from . import _lib
from ._lib import (ACT_ELU, ACT_GELU_ERF, ACT_GELU_TANH, ACT_LEAKY_RELU, ACT_MISH, ACT_NONE,
                   ACT_SILU, BCT, BF16, BIAS_NE0, BIAS_NE1, BTC, F16, F32)

_TORCH_TO_CBX = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
_ACTS = {None: ACT_NONE, "none": ACT_NONE, "mish": ACT_MISH, "silu": ACT_SILU,
         "gelu": ACT_GELU_TANH, "gelu_tanh": ACT_GELU_TANH, "gelu_erf": ACT_GELU_ERF,
         "leaky_relu": ACT_LEAKY_RELU, "elu": ACT_ELU}
_LAYOUTS = {"BCT": BCT, "BTC": BTC}


def _cbx_type(t: torch.Tensor) -> int:
    try:
        return _TORCH_TO_CBX[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype} (f32, f16, bf16)") from None


def _on_tensor_device(fn):
    """Run a wrapper with its first tensor's device current.  The library
    takes its per-device state (SM count, occupancy, error word) from the
    current device, and the stream comes from the tensor's device, so the two
    must agree; the switch is skipped when they already do."""
    @functools.wraps(fn)
    def wrapper(*args, **kw):
        t = args[0] if args else next(iter(kw.values()), None)
        if (isinstance(t, torch.Tensor) and t.is_cuda
                and t.device.index != torch.cuda.current_device()):
            with torch.cuda.device(t.device):
                return fn(*args, **kw)
        return fn(*args, **kw)
    return wrapper


def _dev(t: torch.Tensor | None, name: str, dtype=None):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libcbx_ops has no CPU path)")
    if t.device.index != torch.cuda.current_device():
        raise ValueError(f"{name} is on {t.device}, the call runs on "
                         f"cuda:{torch.cuda.current_device()}: all tensors of a call must "
                         "share its device")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    return ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _act(act) -> int:
    if isinstance(act, int):
        return act
    try:
        return _ACTS[act]
    except KeyError:
        raise ValueError(f"unknown act {act!r}") from None


def _layout(layout) -> int:
    if isinstance(layout, int):
        return layout
    try:
        return _LAYOUTS[layout]
    except KeyError:
        raise ValueError(f"unknown layout {layout!r} (BCT or BTC)") from None


# ------------------------------------------------------------------ gather --

@_on_tensor_device
def embed_gather_add(tok_table: torch.Tensor, ids: torch.Tensor,
                     pos_table: torch.Tensor | None = None, pos_ids: torch.Tensor | None = None,
                     n_past: int = 0, out_dtype: torch.dtype = torch.float32,
                     err_word: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i] = tok_table[ids[i]] + pos_table[pos_ids[i] or n_past + i] (t3.cpp:440-455)."""
    if ids.dtype != torch.int32:
        raise TypeError("ids must be int32")
    n_rows, hidden = ids.numel(), tok_table.shape[-1]
    if out is None:
        out = torch.empty((n_rows, hidden), dtype=out_dtype, device=ids.device)
    _lib.call("cbx_embed_gather_add", _dev(tok_table, "tok_table"), _cbx_type(tok_table),
              tok_table.shape[0], _dev(pos_table, "pos_table"),
              _cbx_type(pos_table) if pos_table is not None else F32,
              pos_table.shape[0] if pos_table is not None else 0, _dev(ids, "ids"),
              _dev(pos_ids, "pos_ids", torch.int32), int(n_past), n_rows, hidden,
              _dev(out, "out"), _cbx_type(out), _dev(err_word, "err_word", torch.int32),
              _stream(ids))
    return out


@_on_tensor_device
def embed_gather_add_batched(tok_table: torch.Tensor, ids: torch.Tensor,
                             pos_table: torch.Tensor | None = None, n_past: int = 0,
                             out_dtype: torch.dtype = torch.float32,
                             err_word: torch.Tensor | None = None,
                             out: torch.Tensor | None = None) -> torch.Tensor:
    """A batch of utterances at the same positions: ids [B, T] ->
    out[b, t] = tok_table[ids[b, t]] + pos_table[n_past + t] (t3.cpp:440-455
    per utterance, one launch for the batch).  Returns [B, T, hidden]."""
    if ids.dtype != torch.int32:
        raise TypeError("ids must be int32")
    if ids.dim() != 2:
        raise ValueError(f"ids must be [n_batch, seq_len], got shape {tuple(ids.shape)}")
    n_batch, seq_len = ids.shape
    hidden = tok_table.shape[-1]
    if pos_table is not None and pos_table.shape[-1] != hidden:
        raise ValueError("pos_table and tok_table differ in hidden size")
    if out is None:
        out = torch.empty((n_batch, seq_len, hidden), dtype=out_dtype, device=ids.device)
    elif out.numel() != n_batch * seq_len * hidden:
        raise ValueError(f"out holds {out.numel()} values, needs {n_batch * seq_len * hidden}")
    _lib.call("cbx_embed_gather_add_batched", _dev(tok_table, "tok_table"), _cbx_type(tok_table),
              tok_table.shape[0], _dev(pos_table, "pos_table"),
              _cbx_type(pos_table) if pos_table is not None else F32,
              pos_table.shape[0] if pos_table is not None else 0, _dev(ids, "ids"),
              n_batch, seq_len, int(n_past), hidden, _dev(out, "out"), _cbx_type(out),
              _dev(err_word, "err_word", torch.int32), _stream(ids))
    return out


@_on_tensor_device
def t3_embed_sequence(tok_table: torch.Tensor, tok_ids: torch.Tensor,
                      pos_table: torch.Tensor | None = None, n_past: int = 0,
                      cond: torch.Tensor | None = None, prompt_table: torch.Tensor | None = None,
                      prompt_ids: torch.Tensor | None = None,
                      out_dtype: torch.dtype = torch.float32,
                      err_word: torch.Tensor | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """The T3 prefill input sequence (t3.cpp:428-455) in one pass:
    [cond rows (f32 [n_cond, H]) ; prompt_table[prompt_ids] ; tok_table[tok_ids]]
    + pos_table[n_past + i].  Returns [n_cond + n_prompt + n_tok, H]."""
    for name, t in (("tok_ids", tok_ids), ("prompt_ids", prompt_ids)):
        if t is not None and t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32")
    if (prompt_ids is None) != (prompt_table is None):
        raise ValueError("prompt_table and prompt_ids go together")
    hidden = tok_table.shape[-1]
    n_cond = 0 if cond is None else cond.reshape(-1, hidden).shape[0]
    if cond is not None and cond.numel() != n_cond * hidden:
        raise ValueError(f"cond holds {cond.numel()} values, not a multiple of hidden {hidden}")
    n_prompt = 0 if prompt_ids is None else prompt_ids.numel()
    if prompt_table is not None and prompt_table.shape[-1] != hidden:
        raise ValueError("prompt_table and tok_table differ in hidden size")
    n_tok = tok_ids.numel()
    if out is None:
        out = torch.empty((n_cond + n_prompt + n_tok, hidden), dtype=out_dtype,
                          device=tok_table.device)
    _lib.call("cbx_t3_embed_sequence", _dev(cond, "cond", torch.float32), n_cond,
              _dev(prompt_table, "prompt_table"),
              _cbx_type(prompt_table) if prompt_table is not None else F32,
              prompt_table.shape[0] if prompt_table is not None else 0,
              _dev(prompt_ids, "prompt_ids"), n_prompt,
              _dev(tok_table, "tok_table"), _cbx_type(tok_table), tok_table.shape[0],
              _dev(tok_ids, "tok_ids"), n_tok, _dev(pos_table, "pos_table"),
              _cbx_type(pos_table) if pos_table is not None else F32,
              pos_table.shape[0] if pos_table is not None else 0, int(n_past), hidden,
              _dev(out, "out"), _cbx_type(out), _dev(err_word, "err_word", torch.int32),
              _stream(tok_table))
    return out


@_on_tensor_device
def t3_embed_sequence_batched(tok_table: torch.Tensor, tok_ids: torch.Tensor,
                              pos_table: torch.Tensor | None = None, n_past: int = 0,
                              cond: torch.Tensor | None = None,
                              prompt_table: torch.Tensor | None = None,
                              prompt_ids: torch.Tensor | None = None,
                              out_dtype: torch.dtype = torch.float32,
                              err_word: torch.Tensor | None = None,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """t3_embed_sequence for a batch of utterances in one launch: tok_ids
    [B, n_tok], prompt_ids [B, n_prompt], cond [B, n_cond, H] (or [B, H]).
    Returns [B, n_cond + n_prompt + n_tok, H]."""
    for name, t in (("tok_ids", tok_ids), ("prompt_ids", prompt_ids)):
        if t is not None and (t.dtype != torch.int32 or t.dim() != 2):
            raise TypeError(f"{name} must be an int32 [n_batch, n] tensor")
    if (prompt_ids is None) != (prompt_table is None):
        raise ValueError("prompt_table and prompt_ids go together")
    B, n_tok = tok_ids.shape
    hidden = tok_table.shape[-1]
    n_prompt = 0 if prompt_ids is None else prompt_ids.shape[1]
    if prompt_ids is not None and prompt_ids.shape[0] != B:
        raise ValueError("prompt_ids and tok_ids differ in batch size")
    if prompt_table is not None and prompt_table.shape[-1] != hidden:
        raise ValueError("prompt_table and tok_table differ in hidden size")
    n_cond = 0
    if cond is not None and B * hidden > 0:
        if cond.numel() % (B * hidden):
            raise ValueError(f"cond holds {cond.numel()} values, not a multiple of B * hidden")
        n_cond = cond.numel() // (B * hidden)
    n = n_cond + n_prompt + n_tok
    if out is None:
        out = torch.empty((B, n, hidden), dtype=out_dtype, device=tok_table.device)
    elif out.numel() != B * n * hidden:
        raise ValueError(f"out holds {out.numel()} values, needs {B * n * hidden}")
    _lib.call("cbx_t3_embed_sequence_batched", _dev(cond, "cond", torch.float32), n_cond,
              _dev(prompt_table, "prompt_table"),
              _cbx_type(prompt_table) if prompt_table is not None else F32,
              prompt_table.shape[0] if prompt_table is not None else 0,
              _dev(prompt_ids, "prompt_ids"), n_prompt,
              _dev(tok_table, "tok_table"), _cbx_type(tok_table), tok_table.shape[0],
              _dev(tok_ids, "tok_ids"), n_tok, _dev(pos_table, "pos_table"),
              _cbx_type(pos_table) if pos_table is not None else F32,
              pos_table.shape[0] if pos_table is not None else 0, int(n_past), hidden, B,
              _dev(out, "out"), _cbx_type(out), _dev(err_word, "err_word", torch.int32),
              _stream(tok_table))
    return out


# --------------------------------------------------------------- layernorm --

@_on_tensor_device
def add_layernorm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor | None,
                  bias: torch.Tensor | None, eps: float = 1e-5, out_dtype=None,
                  return_sum: bool = False, out: torch.Tensor | None = None,
                  sum_out: torch.Tensor | None = None):
    """y = LN(x + residual) * weight + bias over the last dim (t3.cpp:528-532).

    Returns y, or (y, s) with s = x + residual in x's dtype when return_sum."""
    hidden = x.shape[-1]
    n_rows = x.numel() // hidden if hidden else 0
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    if return_sum and sum_out is None:
        sum_out = torch.empty_like(x)
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise ValueError("residual must match x in shape and dtype")
    _lib.call("cbx_add_layernorm", _dev(x, "x"), _dev(residual, "residual"), _cbx_type(x), 0,
              _dev(weight, "weight", torch.float32), _dev(bias, "bias", torch.float32),
              float(eps), n_rows, hidden, _dev(sum_out, "sum_out"), _dev(out, "out"),
              _cbx_type(out), 0, _stream(x))
    return (out, sum_out) if return_sum else out


@_on_tensor_device
def layer_norm(x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None,
               eps: float = 1e-5) -> torch.Tensor:
    """layer_norm(ctx, x, w, b, eps) of cfm_decoder.cpp:29-33 / flow_encoder.cpp:58-62."""
    return add_layernorm(x, None, weight, bias, eps)


@_on_tensor_device
def layernorm_channels(x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None,
                       eps: float = 1e-5, mask: torch.Tensor | None = None, layout="BCT",
                       act="mish", out: torch.Tensor | None = None) -> torch.Tensor:
    """CausalBlock1D tail act(LN_C(x) * w + b) * mask (cfm_decoder.cpp:144-148).

    x: f32 [B, C, T] (layout "BCT") or [B, T, C] ("BTC"); mask: f32 [B, T]."""
    lay = _layout(layout)
    if x.dim() != 3:
        raise ValueError("x must be 3-D")
    B, C, T = (x.shape[0], x.shape[1], x.shape[2]) if lay == BCT else (x.shape[0], x.shape[2],
                                                                       x.shape[1])
    if out is None:
        out = torch.empty_like(x)
    _lib.call("cbx_layernorm_channels", _dev(x, "x", torch.float32),
              _dev(weight, "weight", torch.float32), _dev(bias, "bias", torch.float32),
              float(eps), _dev(mask, "mask", torch.float32), B, C, T, lay, _act(act),
              _dev(out, "out", torch.float32), _stream(x))
    return out


@_on_tensor_device
def causal_block1d_tail(x: torch.Tensor, conv_bias: torch.Tensor | None,
                        weight: torch.Tensor | None, bias: torch.Tensor | None,
                        eps: float = 1e-5, mask: torch.Tensor | None = None, act="mish",
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """The causal conv's epilogue and the CausalBlock1D tail in one pass
    (cfm_decoder.cpp:114-115, :144-148): act(LN_C(x + conv_bias) * w + b) * mask.

    x: f32 [B, C, T] (the conv GEMM's output); returns f32 [B, T, C] (the
    engine's (C, T) layout); mask: f32 [B, T]."""
    if x.dim() != 3:
        raise ValueError("x must be 3-D")
    B, C, T = x.shape
    if out is None:
        out = torch.empty(B, T, C, dtype=torch.float32, device=x.device)
    if tuple(out.shape) != (B, T, C):
        raise ValueError("out must be [B, T, C]")
    _lib.call("cbx_causal_block1d_tail", _dev(x, "x", torch.float32),
              _dev(conv_bias, "conv_bias", torch.float32), _dev(weight, "weight", torch.float32),
              _dev(bias, "bias", torch.float32), float(eps), _dev(mask, "mask", torch.float32),
              B, C, T, _act(act), _dev(out, "out", torch.float32), _stream(x))
    return out


# -------------------------------------------------------------- activations --

def _unary(fn: str, x: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    if out.dtype != x.dtype or out.numel() != x.numel():
        raise ValueError("out must match x")
    _lib.call(fn, _dev(x, "x"), _dev(out, "out"), x.numel(), _cbx_type(x), _stream(x))
    return out


@_on_tensor_device
def gelu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_gelu (GELU-tanh) of t3.cpp:537."""
    return _unary("cbx_gelu_tanh", x, out)


@_on_tensor_device
def silu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_silu of cfm_decoder.cpp:466 / flow_encoder.cpp:402."""
    return _unary("cbx_silu", x, out)


@_on_tensor_device
def mish(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """mish() of cfm_decoder.cpp:36-38."""
    return _unary("cbx_mish", x, out)


@_on_tensor_device
def gelu_erf(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_gelu_erf (exact GELU) of cfm_decoder.cpp:239 / s3enc.cpp:177."""
    return _unary("cbx_gelu_erf", x, out)


# ----------------------------------------------------- epilogue neighbours --

@_on_tensor_device
def bias_act(x: torch.Tensor, bias: torch.Tensor | None = None, act=None, axis: str = "ne0",
             act_param: float = 0.0, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = act(x + bias) over rows of x.shape[-1] elements.

    axis "ne0": bias[j] along the last dim (t3.cpp:536-537 fc bias + GELU);
    axis "ne1": bias[row % len(bias)] per row (conv bias on (T, C),
    cfm_decoder.cpp:114).  act: None, "gelu", "gelu_erf", "silu", "mish",
    "elu", "leaky_relu" (slope act_param; hift_vocoder.cpp:686, :748)."""
    hidden = x.shape[-1]
    n_rows = x.numel() // hidden if hidden else 0
    ax = {"ne0": BIAS_NE0, "ne1": BIAS_NE1}[axis]
    if out is None:
        out = torch.empty_like(x)
    if out.dtype != x.dtype or out.numel() != x.numel():
        raise ValueError("out must match x")
    _lib.call("cbx_bias_act", _dev(x, "x"), _dev(out, "out"), _cbx_type(x), n_rows, hidden,
              _dev(bias, "bias", torch.float32), ax,
              bias.numel() if bias is not None else 0, _act(act), float(act_param), _stream(x))
    return out


@_on_tensor_device
def sum3_scale(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, scale: float = 1.0 / 3.0,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """((a + b) + c) * scale: HiFT's three-ResBlock average (hift_vocoder.cpp:733-739)."""
    if not (a.shape == b.shape == c.shape and a.dtype == b.dtype == c.dtype):
        raise ValueError("a, b, c must match")
    if out is None:
        out = torch.empty_like(a)
    _lib.call("cbx_sum3_scale", _dev(a, "a"), _dev(b, "b"), _dev(c, "c"), float(scale),
              _dev(out, "out"), a.numel(), _cbx_type(a), _stream(a))
    return out


# --------------------------------------------------------------- timesteps --

def sinusoid_freqs(dim: int) -> np.ndarray:
    """Host frequency table of cfm_decoder.cpp:52-56 (f32 [dim // 2])."""
    out = np.empty(dim // 2, np.float32)
    _lib.call("cbx_sinusoid_freqs", int(dim), out.ctypes.data_as(ctypes.c_void_p))
    return out


@_on_tensor_device
def sinusoidal_pos_emb(t: torch.Tensor, dim: int = 320, scale: float = 1000.0, act=None,
                       freqs: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """[n_t, dim] = [sin(a), cos(a)], a = (scale t) freq (cfm_decoder.cpp:49-62), + SiLU."""
    if freqs is None:
        freqs = torch.from_numpy(sinusoid_freqs(dim)).to(t.device)
    n_t = t.numel()
    if out is None:
        out = torch.empty((n_t, dim), dtype=torch.float32, device=t.device)
    _lib.call("cbx_timestep_embed", _dev(t, "t", torch.float32), n_t,
              _dev(freqs, "freqs", torch.float32), int(dim), float(scale), _act(act),
              _dev(out, "out", torch.float32), _stream(t))
    return out


# ------------------------------------------------------------------- snake --

def snake_alpha_inv(alpha: np.ndarray, eps: float = 1e-9) -> np.ndarray:
    """Host 1 / (alpha + eps) in f32 (hift_vocoder.cpp:419-420)."""
    a = np.ascontiguousarray(alpha, np.float32)
    inv = np.empty_like(a)
    _lib.call("cbx_snake_alpha_inv", a.ctypes.data_as(ctypes.c_void_p), a.size, float(eps),
              inv.ctypes.data_as(ctypes.c_void_p))
    return inv


@_on_tensor_device
def snake(x: torch.Tensor, alpha: torch.Tensor, alpha_inv: torch.Tensor | None = None,
          eps: float = 1e-9, layout="BCT", out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x + sin^2(alpha x) * alpha_inv (hift_vocoder.cpp:64-73).

    x: f32 [B, C, T] ("BCT") or [B, T, C] ("BTC"); alpha, alpha_inv: f32 [C]."""
    lay = _layout(layout)
    shape = x.shape
    x3 = x.unsqueeze(0) if x.dim() == 2 else x          # [C, T] / [T, C] -> one item
    if x3.dim() != 3:
        raise ValueError("x must be 2-D or 3-D")
    B, C, T = (x3.shape[0], x3.shape[1], x3.shape[2]) if lay == BCT else (
        x3.shape[0], x3.shape[2], x3.shape[1])
    if out is None:
        out = torch.empty_like(x)
    if out.shape != shape:
        raise ValueError("out must match x")
    _lib.call("cbx_snake", _dev(x, "x", torch.float32), _dev(alpha, "alpha", torch.float32),
              _dev(alpha_inv, "alpha_inv", torch.float32), float(eps), B, C, T, lay,
              _dev(out, "out", torch.float32), _stream(x))
    return out


# ------------------------------------------------------------- HiFT DSP --

NSF_HARMONICS = 9


def hann_window(n_fft: int = 16) -> np.ndarray:
    """Host periodic Hann window, the engine's f32 expression (hift_vocoder.cpp:429-434)."""
    out = np.empty(n_fft, np.float32)
    _lib.call("cbx_hann_window", int(n_fft), out.ctypes.data_as(ctypes.c_void_p))
    return out


@_on_tensor_device
def nsf_source(f0: torch.Tensor, upsample: int, phase: torch.Tensor, noise: torch.Tensor,
               lin_w, lin_b: float = 0.0, sampling_rate: int = 24000,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """HiFT harmonic source (hift_vocoder.cpp:853-965) with explicit phase and noise.

    f0: f32 [B, n_mel] (or [n_mel]); phase: f32 [B, 9]; noise: f32 [B, 9, n_mel * upsample];
    lin_w: the 9 l_linear weights (host sequence); returns f32 [B, n_mel * upsample]."""
    f2 = f0.unsqueeze(0) if f0.dim() == 1 else f0
    B, n_mel = f2.shape
    T = n_mel * int(upsample)
    if phase.numel() != B * NSF_HARMONICS or noise.numel() != B * NSF_HARMONICS * T:
        raise ValueError("phase must hold B*9 and noise B*9*n_mel*upsample values")
    w = np.ascontiguousarray(np.asarray(lin_w, np.float32).reshape(-1))
    if w.size != NSF_HARMONICS:
        raise ValueError("lin_w must hold 9 weights")
    if out is None:
        out = torch.empty((B, T), dtype=torch.float32, device=f0.device)
    _lib.call("cbx_nsf_source", _dev(f2, "f0", torch.float32), B, n_mel, int(upsample),
              int(sampling_rate), _dev(phase, "phase", torch.float32),
              _dev(noise, "noise", torch.float32), w.ctypes.data_as(ctypes.c_void_p),
              float(lin_b), _dev(out, "out", torch.float32), _stream(f0))
    return out


@_on_tensor_device
def stft(audio: torch.Tensor, n_fft: int = 16, hop: int = 4, window: torch.Tensor | None = None,
         layout="BTC", out: torch.Tensor | None = None) -> torch.Tensor:
    """Centered STFT (hift_vocoder.cpp:465-498) of f32 audio [B, T] (or [T]).

    BTC -> [B, T_stft, 2*nb] (real bins then imag bins per frame); BCT -> [B, 2*nb, T_stft]."""
    lay = _layout(layout)
    a2 = audio.unsqueeze(0) if audio.dim() == 1 else audio
    B, T = a2.shape
    if window is None:
        window = torch.from_numpy(hann_window(n_fft)).to(audio.device)
    nb = n_fft // 2 + 1
    Ts = 1 + T // hop
    if out is None:
        shape = (B, Ts, 2 * nb) if lay == BTC else (B, 2 * nb, Ts)
        out = torch.empty(shape, dtype=torch.float32, device=audio.device)
    _lib.call("cbx_stft", _dev(a2, "audio", torch.float32), B, T, int(n_fft), int(hop),
              _dev(window, "window", torch.float32), lay, _dev(out, "out", torch.float32),
              _stream(audio))
    return out


@_on_tensor_device
def istft_post(post: torch.Tensor, n_fft: int = 16, hop: int = 4,
               window: torch.Tensor | None = None, layout="BTC", audio_limit: float = 0.99,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """HiFT output tail (hift_vocoder.cpp:787-829): conv_post channels -> magnitude / phase ->
    centered iSTFT -> clamp.  post: f32 BTC [B, T_f, 2*nb] or BCT [B, 2*nb, T_f] (2-D: one
    item); returns f32 [B, (T_f - 1) * hop]."""
    lay = _layout(layout)
    p3 = post.unsqueeze(0) if post.dim() == 2 else post
    B = p3.shape[0]
    Tf = p3.shape[1] if lay == BTC else p3.shape[2]
    if window is None:
        window = torch.from_numpy(hann_window(n_fft)).to(post.device)
    if out is None:
        out = torch.empty((B, (Tf - 1) * hop), dtype=torch.float32, device=post.device)
    _lib.call("cbx_istft_post", _dev(p3, "post", torch.float32), B, Tf, int(n_fft), int(hop),
              _dev(window, "window", torch.float32), lay, float(audio_limit),
              _dev(out, "out", torch.float32), _stream(post))
    return out


# ------------------------------------------------------- T3 QKV epilogue --

@_on_tensor_device
def qkv_kv_append(qkv: torch.Tensor, bias: torch.Tensor | None, cache_k: torch.Tensor,
                  cache_v: torch.Tensor, positions: torch.Tensor | None = None,
                  pos_offset: int = 0, slab_stride: int = 0, max_context: int | None = None,
                  err: torch.Tensor | None = None, with_q: bool = True):
    """qkv bias add + Q + KV-cache writes (t3.cpp:465-489).

    qkv: f32 [n_rows, 3D]; bias: f32 [3D] or None; cache_k / cache_v: f32 / f16 / bf16
    buffers addressed as cache[r * slab_stride + pos * D + i]; positions: int32 [n_rows]
    (None: pos_offset + r).  Returns (q [n_rows, D] f32 or None, err int32 [1] device)."""
    if qkv.dim() != 2:
        raise ValueError(f"qkv must be 2-D [n_rows, 3D], got shape {tuple(qkv.shape)}")
    n_rows, D3 = qkv.shape
    if D3 % 3:
        raise ValueError(f"qkv's row length {D3} is not a multiple of 3")
    D = D3 // 3
    if max_context is None:
        raise ValueError("max_context required")
    max_context, slab_stride = int(max_context), int(slab_stride)
    if max_context <= 0 or slab_stride < 0:
        raise ValueError(f"max_context {max_context} / slab_stride {slab_stride}")
    if cache_k.dtype != cache_v.dtype:
        raise TypeError("cache_k and cache_v must share a dtype")
    # The kernel writes cache[r * slab_stride + pos * D + i] for pos in
    # [0, max_context): every such element must lie inside both caches, and
    # per-row slabs must not overlap.
    if n_rows > 1 and slab_stride and slab_stride < max_context * D:
        raise ValueError(f"slab_stride {slab_stride} < max_context * D = {max_context * D}: "
                         "the rows' cache slabs would overlap")
    need = (n_rows - 1) * slab_stride + max_context * D if n_rows else 0
    if cache_k.numel() != cache_v.numel() or cache_k.numel() < need:
        raise ValueError(f"caches hold {cache_k.numel()} / {cache_v.numel()} elements; "
                         f"{n_rows} rows at slab_stride {slab_stride} and max_context "
                         f"{max_context} need {need} in each")
    if positions is not None and positions.numel() < n_rows:
        raise ValueError(f"positions has {positions.numel()} entries for {n_rows} rows")
    if bias is not None and bias.numel() != D3:
        raise ValueError(f"bias has {bias.numel()} entries, expected 3D = {D3}")
    if err is not None and err.numel() < 1:
        raise ValueError("err must hold one int32")
    q = torch.empty((n_rows, D), dtype=torch.float32, device=qkv.device) if with_q else None
    if err is None:
        err = torch.zeros(1, dtype=torch.int32, device=qkv.device)
    _lib.call("cbx_qkv_kv_append", _dev(qkv, "qkv", torch.float32), D3,
              _dev(bias, "bias", torch.float32), n_rows, D,
              _dev(positions, "positions", torch.int32), int(pos_offset),
              _dev(cache_k, "cache_k"), _dev(cache_v, "cache_v"), _cbx_type(cache_k),
              int(slab_stride), int(max_context), _dev(q, "q", torch.float32),
              _dev(err, "err", torch.int32), _stream(qkv))
    return q, err
