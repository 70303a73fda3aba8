"""Batched multi-stream T3 decode step, caller side.

The engine decodes one stream at a time (chatterbox-cpp/src/t3.cpp:297-328:
append_speech -> forward_impl per token).  This module runs one decode step
for B independent streams at once: each stream contributes one new token at
its own position, with its own KV-cache slab.  The per-layer order follows
forward_impl (t3.cpp:459-546):

    LN1 -> QKV GEMM -> qkv bias + Q + KV-cache append -> attention over the
    stream's cache -> out GEMM (+ bias) -> attn_residual = out + h -> LN2 ->
    fc GEMM -> fc bias + GELU -> proj GEMM (+ bias) -> h = proj + attn_residual

and ends with the final LayerNorm.  The elementwise steps are libcbx_ops
kernels (called through the C ABI), with each residual add fused into the
next LayerNorm.  The GEMMs are cuBLAS (torch.mm / torch.addmm) and the
attention is torch's scaled_dot_product_attention: both are outside this
library.  Everything is enqueued on the current CUDA stream and allocates
from torch's caching allocator, so a whole step can be captured in one CUDA
graph and replayed with new positions.

A stream whose position is outside [0, max_context) gets no K / V write; the
kernel raises a flag in the model's device error word instead.  ``step``
reads that word after an eager step and raises ``PositionOutOfRange``; when
the step is captured in a CUDA graph the caller calls ``check_errors()``
after each replay.

Weights are random (this repository ships no checkpoints); shapes follow
T3's GPT-2-style blocks (hidden 1024, 16 heads, FFN 4096).
"""
from __future__ import annotations

import torch

from . import ops


class PositionOutOfRange(RuntimeError):
    """A stream's position was outside [0, max_context): its K / V row was not
    written, so the step's attention ran over a stale cache."""


class T3BatchedDecode:
    """B streams, n_layers blocks, KV cache [n_layers][B][max_context][D]."""

    def __init__(self, n_layers: int, B: int, max_context: int, D: int = 1024, H: int = 16,
                 F: int = 4096, cache_dtype=torch.float32, device="cuda", seed: int = 0,
                 eps: float = 1e-5):
        if D % H:
            raise ValueError("D must be a multiple of H")
        self.L, self.B, self.ctx, self.D, self.H, self.F = n_layers, B, max_context, D, H, F
        self.eps = eps
        g = torch.Generator(device=device).manual_seed(seed)

        def w(*shape, std=0.02):
            return torch.randn(*shape, generator=g, device=device) * std

        def ln():
            return 1.0 + 0.1 * torch.randn(D, generator=g, device=device), w(D, std=0.1)

        self.layers = []
        for _ in range(n_layers):
            ln1_w, ln1_b = ln()
            ln2_w, ln2_b = ln()
            self.layers.append(dict(
                ln1_w=ln1_w, ln1_b=ln1_b, qkv_w=w(D, 3 * D), qkv_b=w(3 * D, std=0.1),
                out_w=w(D, D), out_b=w(D, std=0.1), ln2_w=ln2_w, ln2_b=ln2_b,
                fc_w=w(D, F), fc_b=w(F, std=0.1), proj_w=w(F, D), proj_b=w(D, std=0.1)))
        self.lnf_w, self.lnf_b = ln()
        self.cache_k = torch.zeros(n_layers, B, max_context, D, dtype=cache_dtype, device=device)
        self.cache_v = torch.zeros_like(self.cache_k)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    # -- attention over each stream's cache, keys 0..positions[b] -------------
    def _attend(self, q: torch.Tensor, layer: int, positions: torch.Tensor) -> torch.Tensor:
        B, D, H = self.B, self.D, self.H
        hd = D // H
        k = self.cache_k[layer].view(B, self.ctx, H, hd).transpose(1, 2)
        v = self.cache_v[layer].view(B, self.ctx, H, hd).transpose(1, 2)
        qh = q.view(B, H, 1, hd).to(k.dtype)
        keys = torch.arange(self.ctx, device=q.device)
        mask = (keys[None, :] <= positions[:, None].long()).view(B, 1, 1, self.ctx)
        a = torch.nn.functional.scaled_dot_product_attention(qh, k, v, attn_mask=mask)
        return a.reshape(B, D).float()

    def check_errors(self) -> None:
        """Read and clear the device error word (synchronises with the stream);
        raise PositionOutOfRange when a step since the last check saw a
        position outside [0, max_context)."""
        from ._lib import EFLAG_POS_OOB
        flags = int(self.err.item())
        if flags:
            self.err.zero_()
            if flags & EFLAG_POS_OOB:
                raise PositionOutOfRange(
                    f"a stream's position was outside [0, {self.ctx}): its K / V row was not "
                    "written and the step's output is invalid")
            raise RuntimeError(f"decode step device error flags 0x{flags:x}")

    def step(self, x: torch.Tensor, positions: torch.Tensor, check: bool = True) -> torch.Tensor:
        """x: f32 [B, D] token + position embeddings of each stream's new token;
        positions: int32 [B] (each stream's n_past).  Writes the caches and
        returns the final-LN hidden state f32 [B, D].

        With ``check`` (the default) an eager step reads the device error word
        afterwards (one synchronisation) and raises PositionOutOfRange if a
        position was out of range.  Inside CUDA graph capture, or with
        ``check=False``, the caller calls ``check_errors()`` itself."""
        if positions.dtype != torch.int32:
            raise TypeError("positions must be int32")
        out = self._step(x, positions)
        if check and not torch.cuda.is_current_stream_capturing():
            self.check_errors()
        return out

    def _step(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        h = x
        mlp_out = resid = None
        for li, P in enumerate(self.layers):
            if li == 0:
                y1 = ops.layer_norm(h, P["ln1_w"], P["ln1_b"], self.eps)
            else:  # h = proj + attn_residual, fused into LN1 (t3.cpp:545, :465-466)
                y1, h = ops.add_layernorm(mlp_out, resid, P["ln1_w"], P["ln1_b"], self.eps,
                                          return_sum=True)
            qkv = torch.mm(y1, P["qkv_w"])
            q, _ = ops.qkv_kv_append(qkv, P["qkv_b"], self.cache_k[li], self.cache_v[li],
                                     positions=positions, slab_stride=self.ctx * self.D,
                                     max_context=self.ctx, err=self.err)
            a = self._attend(q, li, positions)
            o = torch.addmm(P["out_b"], a, P["out_w"])
            # attn_residual = o + h (t3.cpp:528), fused into LN2
            y2, resid = ops.add_layernorm(o, h, P["ln2_w"], P["ln2_b"], self.eps,
                                          return_sum=True)
            m = ops.bias_act(torch.mm(y2, P["fc_w"]), P["fc_b"], "gelu")
            mlp_out = torch.addmm(P["proj_b"], m, P["proj_w"])
        return ops.add_layernorm(mlp_out, resid, self.lnf_w, self.lnf_b, self.eps)

    # -- the same step with plain torch elementwise ops (the check) -----------
    def step_reference(self, x: torch.Tensor, positions: torch.Tensor, cache_k, cache_v):
        """The step in plain torch fp32 (F.layer_norm, tanh GELU, index writes)
        on separate caches: the reference the library-backed step is tested
        against."""
        B, D = self.B, self.D
        ln = torch.nn.functional.layer_norm
        h = x
        rows = torch.arange(B, device=x.device)
        pos = positions.long()
        for li, P in enumerate(self.layers):
            y1 = ln(h, (D,), P["ln1_w"], P["ln1_b"], self.eps)
            qkv = torch.mm(y1, P["qkv_w"]) + P["qkv_b"]
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            cache_k[li][rows, pos] = k.to(cache_k.dtype)
            cache_v[li][rows, pos] = v.to(cache_v.dtype)
            hd = D // self.H
            kk = cache_k[li].view(B, self.ctx, self.H, hd).transpose(1, 2)
            vv = cache_v[li].view(B, self.ctx, self.H, hd).transpose(1, 2)
            keys = torch.arange(self.ctx, device=x.device)
            mask = (keys[None, :] <= pos[:, None]).view(B, 1, 1, self.ctx)
            a = torch.nn.functional.scaled_dot_product_attention(
                q.reshape(B, self.H, 1, hd).to(kk.dtype), kk, vv, attn_mask=mask)
            a = a.reshape(B, D).float()
            o = torch.addmm(P["out_b"], a, P["out_w"])
            resid = o + h
            y2 = ln(resid, (D,), P["ln2_w"], P["ln2_b"], self.eps)
            m = torch.nn.functional.gelu(torch.mm(y2, P["fc_w"]) + P["fc_b"], approximate="tanh")
            h = torch.addmm(P["proj_b"], m, P["proj_w"]) + resid
        return ln(h, (D,), self.lnf_w, self.lnf_b, self.eps)


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


__all__ = ["PositionOutOfRange", "T3BatchedDecode", "rel_err"]
