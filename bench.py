#!/usr/bin/env python
"""bench.py — throughput of libcbx_ops on the BASELINE configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--no-e2e] [--no-cpu-baseline]

Default workload: BASELINE.json configs[2], the T3 large prefill — 65,536
rows (B=64 x T=1024), hidden 1024, MLP 4096, bf16 activations with f32
statistics: embedding gather-add (token + learned position), residual-add +
LayerNorm, GELU-tanh on [65536, 4096].  One "step" is one pass of that op
stack over the job (1.76 GB of algorithmic bytes, larger than the 126 MB L2);
the three launches are captured in CUDA graphs and replayed.  The other
configs are --workload choices.

Metric: fused layer-op HBM GB/s = algorithmic bytes of the
job's step / step time.  Also reported: rows/s, the roofline of the dominant
kernel (its algorithmic bytes per launch / its mean launch time, measured here
with CUDA events), the end-to-end number through the C ABI with host buffers
(pinned H2D of the step's inputs, the ops, D2H of all outputs, pipelined per
op, and on several ranks the gather of the result rows to rank 0) beside the
copy ceiling of the same traffic, and the CPU oracle timed on the host cores
as the baseline.

Multi-GPU (torchrun, one process per GPU): configs[2] is strong-scaled — the
65,536 rows are split into contiguous per-rank shards, with no collective in
the timed device region; the step time is the max over ranks.  The result
(the LayerNorm output rows) is gathered to rank 0 over NCCL inside the e2e
number, and timed alone as ``gather``.  The other workloads are weak-scaled
(every rank its own batch).

--impl reference times the reference path's CPU implementation (the oracle
restatement of the engine's ggml composition; ggml itself is not buildable
from the reference checkout) on the host cores for the same metric.
"""
from __future__ import annotations

import argparse
import math
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fused layer-op HBM GB/s (% of B200 peak) and rows/s at 1/2/4/8 GPU vs ggml CPU"
FALLBACK_HBM_GBS = 6650.0


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of each kernel from a committed ncu capture
    (profiles/traffic.json: {kernel: {"bytes_per_launch": B, ...}})."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return {}


# ---------------------------------------------------------------- clocks --

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def _one_shot(self):
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"]
            if self.gpu_id is not None:
                cmd += ["-i", self.gpu_id]
            out = subprocess.run(cmd, capture_output=True, text=True, timeout=10).stdout
            self.lines += [l for l in out.splitlines() if l.strip()]
        except Exception:
            pass

    def start(self):
        self._one_shot()
        try:
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "200"]
            if self.gpu_id is not None:
                cmd += ["-i", self.gpu_id]
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)

            def pump():
                for line in self.proc.stdout:
                    if line.strip():
                        self.lines.append(line.strip())
            self._t = threading.Thread(target=pump, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        self._one_shot()
        return self.summary()

    def summary(self):
        rows = []
        for l in self.lines:
            parts = [p.strip() for p in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        reasons = set()
        for _, _, flags in rows:
            for n, f in zip(names[1:], flags[1:]):
                if f.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "samples": len(rows),
                "reasons": sorted(reasons)}


# -------------------------------------------------------------- workloads --

class Launch:
    """One kernel launch of the step: `fn(stream_ptr) -> status`, its kernel
    group and its algorithmic bytes."""

    __slots__ = ("group", "fn", "nbytes")

    def __init__(self, group, fn, nbytes):
        self.group, self.fn, self.nbytes = group, fn, nbytes


def _check(rc, L):
    if rc != 0:
        raise RuntimeError(f"libcbx_ops call failed: {rc} {L.cbx_last_error().decode()}")


class Workload:
    """Device buffers + the ordered launches of one step.

    chunks: [(inputs, outputs, launches)] for the end-to-end pipeline — the
    per-step activations copied in, the outputs copied back, and the launches
    that consume/produce them.  Weights (tables, gamma, beta, alpha) are
    resident and not copied per step."""

    name = ""
    workload = ""
    dtype = "f32"
    rows = 0
    launches: list[Launch]
    chunks: list

    sets = 1
    strong = False      # True: the job is fixed and sharded across ranks (strong scaling)
    gather = None       # (local rows, rank 0's full buffer, rows per rank): the result gather

    @property
    def bytes_per_step(self):
        return sum(l.nbytes for l in self.launches)

    @property
    def all_sets(self):
        """Launch lists of the rotating input sets (one set when inputs exceed L2)."""
        return getattr(self, "set_launches", None) or [self.launches]


class T3Decode(Workload):
    """24 layers x {add+LN, GELU [B,4096], add+LN}, B = 256, H = 1024."""

    def __init__(self, torch, dev, seed, dt="f32", B=256, H=1024, F=4096, L=24):
        from chatterbox_amdvulkan_b200 import _lib
        self.L = _lib.load()
        self.name = f"t3_decode_{dt}"
        self.dtype = dt
        tdt = torch.float32 if dt == "f32" else torch.bfloat16
        ct = _lib.F32 if dt == "f32" else _lib.BF16
        esz = 4 if dt == "f32" else 2
        self.workload = (f"BASELINE configs[1]: T3 batched decode step, {L} layers x "
                         f"(residual-add+LayerNorm, GELU-tanh [{B},{F}], residual-add+LayerNorm),"
                         f" B={B} streams x 1 token, hidden {H}, "
                         + ("f32" if dt == "f32" else "bf16 activations, f32 statistics"))
        self.rows = B
        self.B, self.H, self.F, self.NL = B, H, F, L
        gen = torch.Generator(device=dev).manual_seed(seed)

        def act(n):
            x = torch.randn(n, generator=gen, device=dev)
            m = torch.rand(n, generator=gen, device=dev) < 0.01
            sgn = torch.where(torch.rand(n, generator=gen, device=dev) < 0.5, -20.0, 20.0)
            return torch.where(m, sgn, x)

        BH, BF = B * H, B * F
        self.d_in, self.d_out, self.gb = [], [], []
        self.launches, self.chunks = [], []
        L_ = self.L
        ln_bytes = 4 * BH * esz + 2 * H * 4
        gelu_bytes = 2 * BF * esz
        for l in range(L):
            din = act(4 * BH + BF).to(tdt)          # [x_a | r_a | x_b | r_b | gelu_in]
            dout = torch.empty(4 * BH + BF, dtype=tdt, device=dev)  # [s_a|y_a|s_b|y_b|gelu_out]
            gb = torch.empty(4 * H, dtype=torch.float32, device=dev)
            gb[0:H] = 1 + 0.1 * torch.randn(H, generator=gen, device=dev)
            gb[H:2 * H] = 0.1 * torch.randn(H, generator=gen, device=dev)
            gb[2 * H:3 * H] = 1 + 0.1 * torch.randn(H, generator=gen, device=dev)
            gb[3 * H:] = 0.1 * torch.randn(H, generator=gen, device=dev)
            self.d_in.append(din)
            self.d_out.append(dout)
            self.gb.append(gb)
            pi, po, pg = din.data_ptr(), dout.data_ptr(), gb.data_ptr()
            xa, ra, xb, rb, gi = (pi + k * BH * esz for k in range(5))
            sa, ya, sb, yb, go = (po + k * BH * esz for k in range(5))
            g1, b1, g2, b2 = (pg + k * H * 4 for k in range(4))
            vp = ctypes.c_void_p

            def ln(x, r, g, b, s, y):
                return lambda st: L_.cbx_add_layernorm(vp(x), vp(r), ct, 0, vp(g), vp(b), 1e-5, B,
                                                       H, vp(s), vp(y), ct, 0, vp(st))

            def gelu(x, y):
                return lambda st: L_.cbx_gelu_tanh(vp(x), vp(y), BF, ct, vp(st))

            lay = [Launch("add_layernorm", ln(xa, ra, g1, b1, sa, ya), ln_bytes),
                   Launch("gelu_tanh", gelu(gi, go), gelu_bytes),
                   Launch("add_layernorm", ln(xb, rb, g2, b2, sb, yb), ln_bytes)]
            self.launches += lay
            self.chunks.append(([din], [dout], lay))

    @staticmethod
    def host_step(dt="f32", B=256, H=1024, F=4096, L=24, seed=7):
        """One layer of config 1 on the CPU oracle per call (host arrays, same
        shapes and distributions), cycling through all L layers' buffers so the
        host streams the step's full working set from DRAM as the GPU does.
        Returns (fn, bytes, rows-equivalent, description)."""
        import oracle as O
        rng = np.random.default_rng(seed)
        t = O.F32 if dt == "f32" else O.BF16

        def act(shape):
            x = rng.standard_normal(shape).astype(np.float32)
            m = rng.random(shape) < 0.01
            x[m] = np.where(rng.random(int(m.sum())) < 0.5, -20.0, 20.0)
            return O.to_type(x, t)

        layers = [(act((B, H)), act((B, H)), act((B, H)), act((B, H)), act((B, F)))
                  for _ in range(L)]
        g = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        b = (0.1 * rng.standard_normal(H)).astype(np.float32)
        esz = 4 if dt == "f32" else 2
        state = [0]

        def fn():
            xa, ra, xb, rb, gi = layers[state[0]]
            state[0] = (state[0] + 1) % L
            O.add_layernorm(xa, ra, g, b, 1e-5, in_t=t, out_t=t)
            O.gelu_tanh(gi, t)
            O.add_layernorm(xb, rb, g, b, 1e-5, in_t=t, out_t=t)

        nbytes = 2 * (4 * B * H * esz + 2 * H * 4) + 2 * B * F * esz
        return fn, nbytes, B / float(L), (f"1 layer per call of config 1, cycling through the "
                                          f"{L} layers' buffers ({B} rows: 2 add+LN + GELU)")


class RotatingWorkload(Workload):
    """Base for configs whose per-step working set fits in L2: `sets` copies of
    the activations are cycled (step k uses set k % sets) so every step reads
    inputs that have left L2."""


def _vp(x):
    return ctypes.c_void_p(x)


class T3Prefill(RotatingWorkload):
    """gather-add (512 ids, f32 tables 6563x1024 / 4096x1024,
    positions 0..511) -> residual add + LN over 1024 -> GELU on [512, 4096]."""

    def __init__(self, torch, dev, seed, N=512, H=1024, F=4096, V=6563, P=4096, sets=5):
        from chatterbox_amdvulkan_b200 import _lib
        L = _lib.load()
        self.name, self.dtype, self.rows, self.sets = "t3_prefill_f32", "f32", N, sets
        self.workload = ("BASELINE configs[0]: T3 prefill layer-op stack f32, T=512: embedding "
                         "gather-add (tables 6563x1024, 4096x1024 N(0,0.02)), residual add + "
                         "LayerNorm over 1024, GELU-tanh [512,4096]")
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.tok = 0.02 * torch.randn((V, H), generator=gen, device=dev)
        self.pos = 0.02 * torch.randn((P, H), generator=gen, device=dev)
        self.gb = torch.cat([1 + 0.1 * torch.randn(H, generator=gen, device=dev),
                             0.1 * torch.randn(H, generator=gen, device=dev)])
        pt, pp, pg = self.tok.data_ptr(), self.pos.data_ptr(), self.gb.data_ptr()
        gather_b = N * H * 4 * 3 + N * 4          # out + tok rows + pos rows + ids
        ln_b = 4 * N * H * 4 + 2 * H * 4
        gelu_b = 2 * N * F * 4
        self.set_launches, self.chunks, self.bufs = [], [], []
        for k in range(sets):
            ids = torch.randint(0, 6561, (N,), generator=gen, device=dev, dtype=torch.int32)
            din = torch.randn(N * H + N * F, generator=gen, device=dev)   # [r | gelu_in]
            dh = torch.empty(N * H, device=dev)                          # gather out = LN x
            dout = torch.empty(2 * N * H + N * F, device=dev)             # [s | y | gelu_out]
            self.bufs += [ids, din, dh, dout]
            pi, pd, ph, po = ids.data_ptr(), din.data_ptr(), dh.data_ptr(), dout.data_ptr()
            lz = [Launch("embed_gather_add",
                         lambda st, pi=pi, ph=ph: L.cbx_embed_gather_add(
                             _vp(pt), 0, V, _vp(pp), 0, P, _vp(pi), None, 0, N, H, _vp(ph), 0,
                             None, _vp(st)), gather_b),
                  Launch("add_layernorm",
                         lambda st, ph=ph, pd=pd, po=po: L.cbx_add_layernorm(
                             _vp(ph), _vp(pd), 0, 0, _vp(pg), _vp(pg + H * 4), 1e-5, N, H,
                             _vp(po), _vp(po + N * H * 4), 0, 0, _vp(st)), ln_b),
                  Launch("gelu_tanh",
                         lambda st, pd=pd, po=po: L.cbx_gelu_tanh(
                             _vp(pd + N * H * 4), _vp(po + 2 * N * H * 4), N * F, 0, _vp(st)),
                         gelu_b)]
            self.set_launches.append(lz)
            self.chunks.append(([ids, din], [dout], lz))
        self.launches = self.set_launches[0]

    @staticmethod
    def host_step(N=512, H=1024, F=4096, V=6563, P=4096, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        tok = (0.02 * rng.standard_normal((V, H))).astype(np.float32)
        pos = (0.02 * rng.standard_normal((P, H))).astype(np.float32)
        ids = rng.integers(0, 6561, N).astype(np.int32)
        r = rng.standard_normal((N, H)).astype(np.float32)
        u = rng.standard_normal((N, F)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        b = (0.1 * rng.standard_normal(H)).astype(np.float32)

        def fn():
            h, _ = O.embed_gather_add(tok, O.F32, ids, pos, O.F32, pos_offset=0)
            O.add_layernorm(h, r, g, b, 1e-5)
            O.gelu_tanh(u)

        nb = N * H * 4 * 3 + N * 4 + 4 * N * H * 4 + 2 * H * 4 + 2 * N * F * 4
        return fn, nb, N, "config 0 step (512 rows)"


class T3PrefillLarge(Workload):
    """65536 rows (B=64 x T=1024), bf16 tables/activations, f32 stats.

    Strong scaling: the job is always the 65536 rows; rank r of N owns rows
    shard_range(65536, N, r).  The token ids are drawn for the whole job from
    one seed and sliced, so every N runs the same job; positions are the
    rows' t = row mod 1024.  The result gathered to rank 0 (``gather``) is the
    LayerNorm output y, the hidden rows the next GEMM reads: rank 0's own block
    is a view of the full [65536, 1024] buffer, the other blocks arrive over
    NCCL."""

    strong = True

    def __init__(self, torch, dev, seed, N=65536, H=1024, F=4096, V=6563, P=4096, rank=0,
                 world=1):
        from chatterbox_amdvulkan_b200 import _lib, shard
        L = _lib.load()
        sh = shard.shard_range(N, world, rank)
        n = sh.size
        self.name, self.dtype, self.rows, self.job_rows = "t3_prefill_large_bf16", "bf16", n, N
        self.workload = ("BASELINE configs[2]: T3 large prefill B=64 x T=1024 (65536 rows), "
                         "hidden 1024, MLP 4096: embedding gather-add (bf16 tables, positions "
                         "t mod 1024), residual-add+LayerNorm and GELU-tanh on bf16, f32 stats")
        bf = torch.bfloat16
        gjob = torch.Generator(device=dev).manual_seed(1000)   # the same on every rank
        self.tok = (0.02 * torch.randn((V, H), generator=gjob, device=dev)).to(bf)
        self.pos = (0.02 * torch.randn((P, H), generator=gjob, device=dev)).to(bf)
        ids_job = torch.randint(0, 6561, (N,), generator=gjob, device=dev, dtype=torch.int32)
        pids_job = torch.arange(N, device=dev, dtype=torch.int32) % 1024
        self.gb = torch.cat([1 + 0.1 * torch.randn(H, generator=gjob, device=dev),
                             0.1 * torch.randn(H, generator=gjob, device=dev)])
        self.ids = ids_job[sh.start:sh.stop].clone()
        self.pids = pids_job[sh.start:sh.stop].clone()
        gen = torch.Generator(device=dev).manual_seed(seed)    # activations: per rank
        self.r = torch.randn((n, H), generator=gen, device=dev).to(bf)
        self.u = torch.randn((n, F), generator=gen, device=dev).to(bf)
        self.h = torch.empty((n, H), dtype=bf, device=dev)
        self.s = torch.empty((n, H), dtype=bf, device=dev)
        self.y_full = torch.empty((N, H), dtype=bf, device=dev) if rank == 0 else None
        self.y = self.y_full[:n] if rank == 0 else torch.empty((n, H), dtype=bf, device=dev)
        self.v = torch.empty((n, F), dtype=bf, device=dev)
        self.gather = (self.y, self.y_full, shard.shard_counts(N, world))
        P_ = lambda t: _vp(t.data_ptr())  # noqa: E731

        # A shard of whole utterances (every N that divides 64) runs the batched
        # gather, which takes the positions from the utterance length instead
        # of a position-id array; other shards pass explicit position ids.
        T = 1024
        batched = sh.start % T == 0 and n % T == 0
        self.gather_call = "cbx_embed_gather_add_batched" if batched else "cbx_embed_gather_add"

        def step_bytes(rows, ids, pids, batched):
            uniq = int(torch.unique(ids).numel()) + int(torch.unique(pids).numel())
            id_arrays = 1 if batched else 2
            gather_b = rows * H * 2 + id_arrays * rows * 4 + uniq * H * 2  # compulsory bytes
            return gather_b, 4 * rows * H * 2 + 2 * H * 4, 2 * rows * F * 2

        gather_b, ln_b, gelu_b = step_bytes(n, self.ids, self.pids, batched)
        # the job's bytes: the whole config on one GPU (every N is measured against it)
        self.job_bytes_per_step = sum(step_bytes(N, ids_job, pids_job, N % T == 0))
        del ids_job, pids_job
        tok, pos, ids, pids, r, u, h, s_, y, v, gb = (self.tok, self.pos, self.ids, self.pids,
                                                     self.r, self.u, self.h, self.s, self.y,
                                                     self.v, self.gb)
        if batched:
            gather = Launch("embed_gather_add", lambda st: L.cbx_embed_gather_add_batched(
                P_(tok), 30, V, P_(pos), 30, P, P_(ids), n // T, T, 0, H, P_(h), 30, None,
                _vp(st)), gather_b)
        else:
            gather = Launch("embed_gather_add", lambda st: L.cbx_embed_gather_add(
                P_(tok), 30, V, P_(pos), 30, P, P_(ids), P_(pids), 0, n, H, P_(h), 30, None,
                _vp(st)), gather_b)
        self.launches = [
            gather,
            Launch("add_layernorm", lambda st: L.cbx_add_layernorm(
                P_(h), P_(r), 30, 0, P_(gb), _vp(gb.data_ptr() + H * 4), 1e-5, n, H, P_(s_),
                P_(y), 30, 0, _vp(st)), ln_b),
            Launch("gelu_tanh", lambda st: L.cbx_gelu_tanh(P_(u), P_(v), n * F, 30, _vp(st)),
                   gelu_b)]
        self.chunks = [([ids] if batched else [ids, pids], [h], self.launches[:1]),
                       ([r], [s_, y], self.launches[1:2]),
                       ([u], [v], self.launches[2:])]

    @staticmethod
    def host_step(rows=1024, H=1024, F=4096, V=6563, P=4096, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        tok = O.to_type((0.02 * rng.standard_normal((V, H))).astype(np.float32), O.BF16)
        pos = O.to_type((0.02 * rng.standard_normal((P, H))).astype(np.float32), O.BF16)
        ids = rng.integers(0, 6561, rows).astype(np.int32)
        pids = (np.arange(rows) % 1024).astype(np.int32)
        r = O.to_type(rng.standard_normal((rows, H)).astype(np.float32), O.BF16)
        u = O.to_type(rng.standard_normal((rows, F)).astype(np.float32), O.BF16)
        g = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        b = (0.1 * rng.standard_normal(H)).astype(np.float32)

        def fn():
            h, _ = O.embed_gather_add(tok, O.BF16, ids, pos, O.BF16, pos_ids=pids, out_t=O.BF16)
            O.add_layernorm(h, r, g, b, 1e-5, in_t=O.BF16, out_t=O.BF16)
            O.gelu_tanh(u, O.BF16)

        nb = rows * H * 2 * 3 + 2 * rows * 4 + 4 * rows * H * 2 + 2 * H * 4 + 2 * rows * F * 2
        return fn, nb, rows, f"{rows} of 65536 rows of config 2"


class T3PrefillSeq(Workload):
    """The engine's T3 prefill input, 64 utterances per step: for each one
    cbx_t3_embed_sequence builds [speaker row ; 150 prompt speech rows ; 873
    text rows] + positions 0..1023 (t3.cpp:428-455), f16 tables as the GGUF
    ships them (text 50276 x 1024, speech 6563 x 1024, positions 8196 x 1024)
    and the engine's f32 output.  One cbx_t3_embed_sequence_batched launch
    for the 64 utterances (a server prefilling a batch of requests); the text
    table (103 MB) does not stay in L2."""

    def __init__(self, torch, dev, seed, B=64, H=1024, n_prompt=150, n_text=873, V=50276,
                 S=6563, P=8196):
        from chatterbox_amdvulkan_b200 import _lib
        L = _lib.load()
        n = 1 + n_prompt + n_text
        self.name, self.dtype, self.rows = "t3_prefill_seq_f16", "f16", B * n
        self.workload = (f"T3 prefill input sequence x {B} utterances: [speaker row ; {n_prompt} "
                         f"prompt speech rows ; {n_text} text rows] + positions 0..{n - 1}, f16 "
                         "tables (text 50276x1024, speech 6563x1024, pos 8196x1024), f32 out, "
                         "one cbx_t3_embed_sequence_batched launch for the batch")
        gen = torch.Generator(device=dev).manual_seed(seed)
        f16 = torch.float16
        self.text = (0.02 * torch.randn((V, H), generator=gen, device=dev)).to(f16)
        self.speech = (0.02 * torch.randn((S, H), generator=gen, device=dev)).to(f16)
        self.pos = (0.02 * torch.randn((P, H), generator=gen, device=dev)).to(f16)
        self.cond = torch.randn((B, H), generator=gen, device=dev)
        self.pids = torch.randint(0, S, (B, n_prompt), generator=gen, device=dev,
                                  dtype=torch.int32)
        self.tids = torch.randint(0, V, (B, n_text), generator=gen, device=dev,
                                  dtype=torch.int32)
        self.out = torch.empty((B, n, H), dtype=torch.float32, device=dev)
        uniq = (int(torch.unique(self.pids).numel()) + int(torch.unique(self.tids).numel())
                + n) * H * 2                                   # distinct table rows
        step_b = B * n * H * 4 + B * (n - 1) * 4 + B * H * 4 + uniq
        self.compulsory = {"out": B * n * H * 4, "ids": B * (n - 1) * 4, "cond": B * H * 4,
                           "distinct_table_rows": uniq}
        vp = _vp
        tx, sp, po, cd, pi, ti, out = (self.text, self.speech, self.pos, self.cond, self.pids,
                                       self.tids, self.out)

        self.launches = [Launch("t3_embed_sequence", lambda st: L.cbx_t3_embed_sequence_batched(
            vp(cd.data_ptr()), 1, vp(sp.data_ptr()), 1, S, vp(pi.data_ptr()), n_prompt,
            vp(tx.data_ptr()), 1, V, vp(ti.data_ptr()), n_text, vp(po.data_ptr()), 1, P, 0, H, B,
            vp(out.data_ptr()), 0, None, vp(st)), step_b)]
        self.chunks = [([self.cond, self.pids, self.tids], [self.out], self.launches)]

    @staticmethod
    def host_step(B=4, H=1024, n_prompt=150, n_text=873, V=50276, S=6563, P=8196, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        text = O.to_type((0.02 * rng.standard_normal((V, H))).astype(np.float32), O.F16)
        speech = O.to_type((0.02 * rng.standard_normal((S, H))).astype(np.float32), O.F16)
        pos = O.to_type((0.02 * rng.standard_normal((P, H))).astype(np.float32), O.F16)
        cond = rng.standard_normal((B, H)).astype(np.float32)
        pids = rng.integers(0, S, (B, n_prompt)).astype(np.int32)
        tids = rng.integers(0, V, (B, n_text)).astype(np.int32)
        n = 1 + n_prompt + n_text

        def fn():
            for b in range(B):
                O.t3_embed_sequence(text, O.F16, tids[b], pos, O.F16, 0, cond[b], speech, O.F16,
                                    pids[b])

        nb = B * (n * H * 4 + (n - 1) * 4 + H * 4 + (n - 1 + n) * H * 2)
        return fn, nb, B * n, f"{B} utterances of the prefill sequence ({n} rows each)"


class CfmOps(RotatingWorkload):
    """LN over C + Mish on [32, 256, 1000] f32 (channel-strided) and
    the sinusoidal timestep embedding (32 t, dim 320, scale 1000) + SiLU."""

    def __init__(self, torch, dev, seed, B=32, C=256, T=1000, dim=320, sets=4):
        from chatterbox_amdvulkan_b200 import _lib, ops
        L = _lib.load()
        self.name, self.dtype, self.rows, self.sets = "cfm_ops_f32", "f32", B * T, sets
        self.workload = ("BASELINE configs[3]: CFM estimator ops on channels-first "
                         "[32,256,1000] f32: LayerNorm over C (eps 1e-5) + Mish; sinusoidal "
                         "timestep embedding (32 t ~ U[0,1], dim 320, scale 1000) + SiLU")
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.gb = torch.cat([1 + 0.1 * torch.randn(C, generator=gen, device=dev),
                             0.1 * torch.randn(C, generator=gen, device=dev)])
        self.freqs = torch.from_numpy(ops.sinusoid_freqs(dim)).to(dev)
        pg, pf = self.gb.data_ptr(), self.freqs.data_ptr()
        n = B * C * T
        self.set_launches, self.chunks, self.bufs = [], [], []
        for k in range(sets):
            x = torch.randn(n, generator=gen, device=dev)
            y = torch.empty(n, device=dev)
            t = torch.rand(B, generator=gen, device=dev)
            e = torch.empty(B * dim, device=dev)
            self.bufs += [x, y, t, e]
            px, py, pt, pe = x.data_ptr(), y.data_ptr(), t.data_ptr(), e.data_ptr()
            lz = [Launch("layernorm_channels",
                         lambda st, px=px, py=py: L.cbx_layernorm_channels(
                             _vp(px), _vp(pg), _vp(pg + C * 4), 1e-5, None, B, C, T, 0, 1,
                             _vp(py), _vp(st)), 2 * n * 4 + 2 * C * 4),
                  Launch("timestep_embed",
                         lambda st, pt=pt, pe=pe: L.cbx_timestep_embed(
                             _vp(pt), B, _vp(pf), dim, 1000.0, 2, _vp(pe), _vp(st)),
                         B * dim * 4 + B * 4)]
            self.set_launches.append(lz)
            self.chunks.append(([x, t], [y, e], lz))
        self.launches = self.set_launches[0]

    @staticmethod
    def host_step(C=256, T=1000, dim=320, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((1, C, T)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
        b = (0.1 * rng.standard_normal(C)).astype(np.float32)
        t = rng.random(1).astype(np.float32)

        def fn():
            O.layernorm_channels(x, g, b, 1e-5, None, O.BCT, O.ACT_MISH)
            O.timestep_embed(t, dim, 1000.0, O.ACT_SILU)

        return fn, 2 * C * T * 4 + 2 * C * 4 + dim * 4 + 4, T, "1 of 32 batch items of config 3"


class CfmActs(RotatingWorkload):
    """SiLU and Mish as standalone nodes (cfm_decoder.cpp:466, :36-38) on the
    config-3 activation shape [32, 256, 1000] f32, each on its own buffers;
    2 rotating input sets (262 MB), so every step reads inputs that left L2."""

    def __init__(self, torch, dev, seed, B=32, C=256, T=1000, sets=2):
        from chatterbox_amdvulkan_b200 import _lib
        L = _lib.load()
        self.name, self.dtype, self.rows, self.sets = "cfm_act_f32", "f32", B * C, sets
        self.workload = ("SiLU and Mish (standalone nodes) on [32,256,1000] f32, the config-3 "
                         "activation shape")
        gen = torch.Generator(device=dev).manual_seed(seed)
        n = B * C * T
        self.set_launches, self.chunks, self.bufs = [], [], []
        for k in range(sets):
            xs, ys = torch.randn(n, generator=gen, device=dev), torch.empty(n, device=dev)
            xm, ym = torch.randn(n, generator=gen, device=dev), torch.empty(n, device=dev)
            self.bufs += [xs, ys, xm, ym]
            lz = [Launch("silu", lambda st, x=xs, y=ys: L.cbx_silu(
                      _vp(x.data_ptr()), _vp(y.data_ptr()), n, 0, _vp(st)), 2 * n * 4),
                  Launch("mish", lambda st, x=xm, y=ym: L.cbx_mish(
                      _vp(x.data_ptr()), _vp(y.data_ptr()), n, 0, _vp(st)), 2 * n * 4)]
            self.set_launches.append(lz)
            self.chunks.append(([xs, xm], [ys, ym], lz))
        self.launches = self.set_launches[0]

    @staticmethod
    def host_step(C=256, T=1000, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((C, T)).astype(np.float32)

        def fn():
            O.silu(x)
            O.mish(x)

        return fn, 4 * C * T * 4, C, "1 of 32 batch items of both activations"


class CfmBlockTail(RotatingWorkload):
    """The causal conv's epilogue + CausalBlock1D tail at configs[3]'s shape:
    conv GEMM output [32, 256, 1000] f32 + conv bias -> LN over C + Mish + mask
    -> [32, 1000, 256] (cfm_decoder.cpp:114-115, :144-148) in one pass."""

    def __init__(self, torch, dev, seed, B=32, C=256, T=1000, sets=4):
        from chatterbox_amdvulkan_b200 import _lib
        L = _lib.load()
        self.name, self.dtype, self.rows, self.sets = "cfm_block_tail_f32", "f32", B * T, sets
        self.workload = ("CFM causal conv epilogue + CausalBlock1D tail at configs[3]'s shape: "
                         "conv output [32,256,1000] f32 + conv bias, transposed to the engine's "
                         "[32,1000,256], LayerNorm over C (eps 1e-5) + Mish + mask")
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.par = torch.cat([0.5 * torch.randn(C, generator=gen, device=dev),
                              1 + 0.1 * torch.randn(C, generator=gen, device=dev),
                              0.1 * torch.randn(C, generator=gen, device=dev)])
        self.mask = (torch.rand(B, T, generator=gen, device=dev) > 0.05).float()
        pp, pm = self.par.data_ptr(), self.mask.data_ptr()
        n = B * C * T
        self.set_launches, self.chunks, self.bufs = [], [], [self.par, self.mask]
        for k in range(sets):
            x = torch.randn(n, generator=gen, device=dev)
            y = torch.empty(n, device=dev)
            self.bufs += [x, y]
            px, py = x.data_ptr(), y.data_ptr()
            lz = [Launch("causal_block1d_tail",
                         lambda st, px=px, py=py: L.cbx_causal_block1d_tail(
                             _vp(px), _vp(pp), _vp(pp + C * 4), _vp(pp + 2 * C * 4), 1e-5,
                             _vp(pm), B, C, T, 1, _vp(py), _vp(st)),
                         2 * n * 4 + 3 * C * 4 + B * T * 4)]
            self.set_launches.append(lz)
            self.chunks.append(([x], [y], lz))
        self.launches = self.set_launches[0]

    @staticmethod
    def host_step(C=256, T=1000, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((1, C, T)).astype(np.float32)
        cb = (0.5 * rng.standard_normal(C)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
        b = (0.1 * rng.standard_normal(C)).astype(np.float32)
        m = (rng.random((1, T)) > 0.05).astype(np.float32)

        def fn():
            O.causal_block1d_tail(x, cb, g, b, 1e-5, m, O.ACT_MISH)

        return fn, 2 * C * T * 4 + 3 * C * 4 + T * 4, T, "1 of 32 batch items"


class HiftSnake(Workload):
    """Snake, B=16 at [256,4000], [128,20000], [64,60000] f32."""

    STAGES = ((256, 4000), (128, 20000), (64, 60000))

    def __init__(self, torch, dev, seed, B=16, layout=0):
        from chatterbox_amdvulkan_b200 import _lib, ops
        L = _lib.load()
        self.name = "hift_snake_f32" if layout == 0 else "hift_snake_btc_f32"
        self.dtype = "f32"
        self.rows = B * sum(c for c, _ in self.STAGES)
        self.workload = ("BASELINE configs[4]: HiFT Snake x + sin^2(ax)/(a+1e-9) f32, B=16 at "
                         "[256,4000], [128,20000], [64,60000]; a = exp(N(0,0.3))" +
                         ("" if layout == 0 else "; the engine's [B][T][C] layout"))
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.launches, self.chunks, self.bufs = [], [], []
        for C, T in self.STAGES:
            x = torch.randn(B * C * T, generator=gen, device=dev)
            y = torch.empty_like(x)
            a = torch.exp(0.3 * torch.randn(C, generator=gen, device=dev))
            ai = torch.from_numpy(ops.snake_alpha_inv(a.cpu().numpy())).to(dev)
            self.bufs += [x, y, a, ai]
            l = Launch(f"snake_c{C}", lambda st, x=x, y=y, a=a, ai=ai, C=C, T=T: L.cbx_snake(
                _vp(x.data_ptr()), _vp(a.data_ptr()), _vp(ai.data_ptr()), 1e-9, B, C, T, layout,
                _vp(y.data_ptr()), _vp(st)), 2 * B * C * T * 4)
            self.launches.append(l)
            self.chunks.append(([x], [y], [l]))

    @staticmethod
    def host_step(seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        xs = []
        for C, T in HiftSnake.STAGES:
            x = rng.standard_normal((1, C, T)).astype(np.float32)
            a = np.exp(0.3 * rng.standard_normal(C)).astype(np.float32)
            xs.append((x, a, O.snake_alpha_inv(a)))

        def fn():
            for x, a, ai in xs:
                O.snake(x, a, ai)

        nb = sum(2 * C * T * 4 for C, T in HiftSnake.STAGES)
        return fn, nb, sum(c for c, _ in HiftSnake.STAGES), "1 of 16 utterances of config 4"


class T3FcEpilogue(Workload):
    """GEMM-epilogue neighbour: T3 FFN fc bias + GELU-tanh (t3.cpp:536-537)
    on the config-2 shape [65536, 4096] bf16, f32 bias."""

    def __init__(self, torch, dev, seed, N=65536, F=4096):
        from chatterbox_amdvulkan_b200 import _lib
        L = _lib.load()
        self.name, self.dtype, self.rows = "t3_fc_epilogue_bf16", "bf16", N
        self.workload = ("GEMM-epilogue neighbour: T3 FFN fc bias + GELU-tanh on "
                         "[65536, 4096] bf16 (config-2 shape), f32 bias")
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.x = torch.randn((N, F), generator=gen, device=dev).to(torch.bfloat16)
        self.y = torch.empty_like(self.x)
        self.b = 0.5 * torch.randn(F, generator=gen, device=dev)
        x, y, b = self.x, self.y, self.b
        self.launches = [Launch("bias_gelu", lambda st: L.cbx_bias_act(
            _vp(x.data_ptr()), _vp(y.data_ptr()), 30, N, F, _vp(b.data_ptr()), 0, F, 3, 0.0,
            _vp(st)), 2 * N * F * 2 + F * 4)]
        self.chunks = [([x], [y], self.launches)]

    @staticmethod
    def host_step(rows=512, F=4096, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        x = O.to_type(rng.standard_normal((rows, F)).astype(np.float32), O.BF16)
        b = (0.5 * rng.standard_normal(F)).astype(np.float32)

        def fn():
            O.bias_act(x, b, O.BIAS_NE0, O.ACT_GELU, 0.0, O.BF16)

        return fn, 2 * rows * F * 2 + F * 4, rows, f"{rows} of 65536 rows"


class S3genEpilogue(Workload):
    """GEMM-epilogue neighbours in S3Gen: exact GELU on the CFM transformer FF hidden
    [32 x 1000, 1024] f32 (cfm_decoder.cpp:239), and per HiFT stage (B=16) the
    three-ResBlock average and the LeakyReLU(0.1) that opens the next stage
    (hift_vocoder.cpp:733-739, :686)."""

    STAGES = ((256, 4000), (128, 20000), (64, 60000))

    def __init__(self, torch, dev, seed, B=16):
        from chatterbox_amdvulkan_b200 import _lib
        L = _lib.load()
        self.name, self.dtype = "s3gen_epilogue_f32", "f32"
        self.rows = 32 * 1000 + B * sum(c for c, _ in self.STAGES)
        self.workload = ("GEMM-epilogue neighbours, f32: GELU-erf on CFM FF hidden "
                         "[32000, 1024]; HiFT ResBlock mean (sum3 x 1/3) + LeakyReLU(0.1) on "
                         "[16,256,4000], [16,128,20000], [16,64,60000]")
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.bufs = []
        n_ff = 32 * 1000 * 1024
        xf = torch.randn(n_ff, generator=gen, device=dev)
        yf = torch.empty_like(xf)
        self.bufs += [xf, yf]
        self.launches = [Launch("gelu_erf", lambda st, xf=xf, yf=yf: L.cbx_gelu_erf(
            _vp(xf.data_ptr()), _vp(yf.data_ptr()), n_ff, 0, _vp(st)), 2 * n_ff * 4)]
        self.chunks = [([xf], [yf], self.launches[:1])]
        for C, T in self.STAGES:
            n = B * C * T
            r = [torch.randn(n, generator=gen, device=dev) for _ in range(3)]
            m = torch.empty(n, device=dev)
            o = torch.empty(n, device=dev)
            self.bufs += r + [m, o]
            l1 = Launch(f"rb_mean_c{C}", lambda st, r=r, m=m, n=n: L.cbx_sum3_scale(
                _vp(r[0].data_ptr()), _vp(r[1].data_ptr()), _vp(r[2].data_ptr()),
                1.0 / 3.0, _vp(m.data_ptr()), n, 0, _vp(st)), 4 * n * 4)
            l2 = Launch(f"leaky_c{C}", lambda st, m=m, o=o, n=n, C=C, T=T: L.cbx_bias_act(
                _vp(m.data_ptr()), _vp(o.data_ptr()), 0, B * C, T, None, 0, 0, 5, 0.1,
                _vp(st)), 2 * n * 4)
            self.launches += [l1, l2]
            self.chunks.append((r, [o], [l1, l2]))

    @staticmethod
    def host_step(seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        xf = rng.standard_normal((1000, 1024)).astype(np.float32)
        st = []
        for C, T in S3genEpilogue.STAGES:
            st.append([rng.standard_normal((C, T)).astype(np.float32) for _ in range(3)])

        def fn():
            O.gelu_erf(xf)
            for r in st:
                m = O.sum3_scale(r[0], r[1], r[2], np.float32(1.0 / 3.0))
                O.bias_act(m, None, O.BIAS_NE0, O.ACT_LEAKY_RELU, 0.1)

        nb = 2 * xf.size * 4 + sum(6 * C * T * 4 for C, T in S3genEpilogue.STAGES)
        return fn, nb, 1000 + sum(c for c, _ in S3genEpilogue.STAGES), \
            "1 of 32 CFM items + 1 of 16 HiFT utterances"


class T3DecodeStep(Workload):
    """The library's share of a real batched T3 decode step (the
    elementwise ops of chatterbox_amdvulkan_b200/decode_step.py) for B = 256
    streams, 24 layers: per layer add + LN1, the QKV epilogue with the KV-cache
    append at each stream's own position (f32 cache [256][ctx 64][1024] per
    layer), add + LN2 and the fc bias + GELU.  The GEMMs and the attention
    between them are cuBLAS / torch and not part of this library's figure."""

    def __init__(self, torch, dev, seed, B=256, D=1024, F=4096, L=24, ctx=64):
        from chatterbox_amdvulkan_b200 import _lib
        L_ = _lib.load()
        self.name, self.dtype, self.rows = "t3_decode_step_f32", "f32", B
        self.workload = (f"elementwise share of a batched T3 decode step, B={B} "
                         f"streams, {L} layers, hidden {D}, FFN {F}: add+LN1, QKV bias + Q + "
                         f"KV-cache append (f32 cache, ctx {ctx}, per-stream positions), add+LN2, "
                         f"fc bias + GELU")
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.launches, self.chunks, self.bufs = [], [], []
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        pos = torch.randint(0, ctx, (B,), generator=gen, device=dev, dtype=torch.int32)
        self.bufs.append(pos)
        perr, ppos = self.err.data_ptr(), pos.data_ptr()
        for _ in range(L):
            def t(*shape):
                return torch.randn(*shape, generator=gen, device=dev)
            mlp, resid, h, y1 = t(B, D), t(B, D), torch.empty(B, D, device=dev), \
                torch.empty(B, D, device=dev)
            qkv, qb, q = t(B, 3 * D), t(3 * D), torch.empty(B, D, device=dev)
            ck = torch.zeros(B, ctx, D, device=dev)
            cv = torch.zeros(B, ctx, D, device=dev)
            o, r2, y2 = t(B, D), torch.empty(B, D, device=dev), torch.empty(B, D, device=dev)
            fc, fb, g = t(B, F), t(F), torch.empty(B, F, device=dev)
            gb = torch.cat([1 + 0.1 * t(D), 0.1 * t(D)])
            self.bufs += [mlp, resid, h, y1, qkv, qb, q, ck, cv, o, r2, y2, fc, fb, g, gb]
            p = {k: v.data_ptr() for k, v in dict(mlp=mlp, resid=resid, h=h, y1=y1, qkv=qkv, qb=qb,
                                                   q=q, ck=ck, cv=cv, o=o, r2=r2, y2=y2, fc=fc,
                                                   fb=fb, g=g, gb=gb).items()}
            lz = [
                Launch("add_layernorm", lambda st, p=p: L_.cbx_add_layernorm(
                    _vp(p["mlp"]), _vp(p["resid"]), 0, 0, _vp(p["gb"]), _vp(p["gb"] + D * 4),
                    1e-5, B, D, _vp(p["h"]), _vp(p["y1"]), 0, 0, _vp(st)), 5 * B * D * 4 + 8 * D),
                Launch("qkv_kv_append", lambda st, p=p: L_.cbx_qkv_kv_append(
                    _vp(p["qkv"]), 3 * D, _vp(p["qb"]), B, D, _vp(ppos), 0, _vp(p["ck"]),
                    _vp(p["cv"]), 0, ctx * D, ctx, _vp(p["q"]), _vp(perr), _vp(st)),
                    B * 3 * D * 4 + 3 * D * 4 + B * 4 + B * D * 4 + 2 * B * D * 4),
                Launch("add_layernorm", lambda st, p=p: L_.cbx_add_layernorm(
                    _vp(p["o"]), _vp(p["h"]), 0, 0, _vp(p["gb"]), _vp(p["gb"] + D * 4), 1e-5, B,
                    D, _vp(p["r2"]), _vp(p["y2"]), 0, 0, _vp(st)), 5 * B * D * 4 + 8 * D),
                Launch("bias_gelu", lambda st, p=p: L_.cbx_bias_act(
                    _vp(p["fc"]), _vp(p["g"]), 0, B, F, _vp(p["fb"]), 0, F, 3, 0.0, _vp(st)),
                    2 * B * F * 4 + F * 4),
            ]
            self.launches += lz
            self.chunks.append(([mlp, resid, qkv, o, fc], [y1, q, y2, g], lz))

    @staticmethod
    def host_step(B=256, D=1024, F=4096, ctx=64, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        r = 16  # 16 of the 256 streams, one layer
        mlp, resid = rng.standard_normal((r, D)).astype(np.float32), \
            rng.standard_normal((r, D)).astype(np.float32)
        qkv, qb = rng.standard_normal((r, 3 * D)).astype(np.float32), \
            rng.standard_normal(3 * D).astype(np.float32)
        o = rng.standard_normal((r, D)).astype(np.float32)
        fc, fb = rng.standard_normal((r, F)).astype(np.float32), \
            rng.standard_normal(F).astype(np.float32)
        g, b = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32), \
            (0.1 * rng.standard_normal(D)).astype(np.float32)
        ck = np.zeros((r, ctx, D), np.float32)
        cv = np.zeros((r, ctx, D), np.float32)
        pos = rng.integers(0, ctx, r).astype(np.int32)

        def fn():
            s, _ = O.add_layernorm(mlp, resid, g, b, 1e-5)
            O.qkv_kv_append(qkv, qb, ck, cv, O.F32, positions=pos, slab_stride=ctx * D,
                            max_context=ctx)
            O.add_layernorm(o, s, g, b, 1e-5)
            O.bias_act(fc, fb, O.BIAS_NE0, O.ACT_GELU)

        nb = 2 * (5 * r * D * 4 + 8 * D) + r * 3 * D * 4 + 3 * D * 4 + r * 4 + 3 * r * D * 4 + \
            2 * r * F * 4 + F * 4
        return fn, nb, r, "16 of 256 streams x 1 of 24 layers of the decode step"


class HiftDsp(Workload):
    """The HiFT host DSP either side of the Snake stack, for B
    utterances of 10 s at 24 kHz (n_mel = 500, upsample 480): the NSF harmonic
    source from f0 with explicit phase / noise (hift_vocoder.cpp:853-965), the
    centered STFT of that source (n_fft 16, hop 4; :465-498, engine row layout)
    and the output tail from conv_post's 18 channels (magnitude / phase,
    iSTFT, clamp; :787-829)."""

    def __init__(self, torch, dev, seed, B=32, n_mel=500, up=480):
        from chatterbox_amdvulkan_b200 import _lib, ops
        L = _lib.load()
        self.name, self.dtype = "hift_dsp_f32", "f32"
        T = n_mel * up
        Tf = T // 4 + 1
        self.rows = B
        self.workload = (f"HiFT NSF source + source STFT + iSTFT output tail, "
                         f"B={B} utterances x 10 s at 24 kHz (n_mel {n_mel}, upsample {up}, "
                         f"n_fft 16, hop 4), f32, explicit phase/noise")
        gen = torch.Generator(device=dev).manual_seed(seed)
        t = torch.arange(n_mel, device=dev, dtype=torch.float32)
        f0 = 150.0 + 60.0 * torch.sin(t[None, :] / 17.0 + torch.rand(B, 1, generator=gen,
                                                                     device=dev) * 6.0)
        f0 = torch.where(torch.rand(B, n_mel, generator=gen, device=dev) < 0.2,
                         torch.zeros_like(f0), f0).contiguous()
        phase = (torch.rand(B, 9, generator=gen, device=dev) * 2 - 1) * math.pi
        noise = torch.randn(B, 9, T, generator=gen, device=dev)
        src = torch.empty(B, T, device=dev)
        spec = torch.empty(B, Tf, 18, device=dev)
        post = torch.cat([torch.randn(B, Tf, 9, generator=gen, device=dev) * 0.9 - 2.0,
                          torch.randn(B, Tf, 9, generator=gen, device=dev) * 2.0], dim=2)
        post = post.contiguous()
        wav = torch.empty(B, T, device=dev)
        win = torch.from_numpy(ops.hann_window(16)).to(dev)
        lw = (0.4 * np.random.default_rng(seed).standard_normal(9)).astype(np.float32)
        self.bufs = [f0, phase, noise, src, spec, post, wav, win]
        self.lw = lw
        pw = lw.ctypes.data_as(ctypes.c_void_p)
        self.launches = [
            Launch("nsf_source", lambda st: L.cbx_nsf_source(
                _vp(f0.data_ptr()), B, n_mel, up, 24000, _vp(phase.data_ptr()),
                _vp(noise.data_ptr()), pw, 0.02, _vp(src.data_ptr()), _vp(st)),
                4 * (B * n_mel + B * 9 + B * 9 * T + B * T)),
            Launch("stft", lambda st: L.cbx_stft(
                _vp(src.data_ptr()), B, T, 16, 4, _vp(win.data_ptr()), 1, _vp(spec.data_ptr()),
                _vp(st)), 4 * (B * T + 16 + B * Tf * 18)),
            Launch("istft_post", lambda st: L.cbx_istft_post(
                _vp(post.data_ptr()), B, Tf, 16, 4, _vp(win.data_ptr()), 1, 0.99,
                _vp(wav.data_ptr()), _vp(st)), 4 * (B * Tf * 18 + 16 + B * (Tf - 1) * 4)),
        ]
        self.chunks = [([f0, phase, noise], [src], self.launches[:1]),
                       ([], [spec], self.launches[1:2]),
                       ([post], [wav], self.launches[2:])]

    @staticmethod
    def host_step(B=16, n_mel=500, up=480, seed=7):
        import oracle as O
        rng = np.random.default_rng(seed)
        T = n_mel * up
        f0 = (150.0 + 60.0 * np.sin(np.arange(n_mel)[None] / 17.0 + rng.random((B, 1)) * 6.0))
        f0 = np.where(rng.random((B, n_mel)) < 0.2, 0.0, f0).astype(np.float32)
        phase = rng.uniform(-np.pi, np.pi, (B, 9)).astype(np.float32)
        noise = rng.standard_normal((B, 9, T)).astype(np.float32)
        lw = (0.4 * rng.standard_normal(9)).astype(np.float32)
        Tf = T // 4 + 1
        post = np.concatenate([rng.normal(-2.0, 0.9, (B, Tf, 9)), rng.normal(0, 2.0, (B, Tf, 9))],
                              axis=2).astype(np.float32)
        win = O.hann_window(16)

        def fn():
            src = O.nsf_source(f0, up, phase, noise, lw, 0.02)
            O.stft(src, 16, 4, win)
            O.istft_post(post, 16, 4, win)

        nb = 4 * (B * n_mel + B * 9 + B * 9 * T + B * T) + 4 * (B * T + 16 + B * Tf * 18) + \
            4 * (B * Tf * 18 + 16 + B * (Tf - 1) * 4)
        return fn, nb, B, f"{B} of 32 utterances of the HiFT DSP step"


WORKLOADS = {
    "t3_decode_f32": (lambda torch, dev, seed: T3Decode(torch, dev, seed, "f32"),
                      lambda: T3Decode.host_step("f32"), "f32"),
    "t3_decode_bf16": (lambda torch, dev, seed: T3Decode(torch, dev, seed, "bf16"),
                       lambda: T3Decode.host_step("bf16"), "bf16"),
    "t3_prefill_f32": (T3Prefill, T3Prefill.host_step, "f32"),
    "t3_prefill_large_bf16": (T3PrefillLarge, T3PrefillLarge.host_step, "bf16"),
    "t3_prefill_seq_f16": (T3PrefillSeq, T3PrefillSeq.host_step, "f16"),
    "cfm_ops_f32": (CfmOps, CfmOps.host_step, "f32"),
    "cfm_block_tail_f32": (CfmBlockTail, CfmBlockTail.host_step, "f32"),
    "cfm_act_f32": (CfmActs, CfmActs.host_step, "f32"),
    "hift_snake_f32": (HiftSnake, HiftSnake.host_step, "f32"),
    "hift_snake_btc_f32": (lambda torch, dev, seed: HiftSnake(torch, dev, seed, layout=1),
                           HiftSnake.host_step, "f32"),
    "t3_fc_epilogue_bf16": (T3FcEpilogue, T3FcEpilogue.host_step, "bf16"),
    "s3gen_epilogue_f32": (S3genEpilogue, S3genEpilogue.host_step, "f32"),
    "hift_dsp_f32": (HiftDsp, HiftDsp.host_step, "f32"),
    "t3_decode_step_f32": (T3DecodeStep, T3DecodeStep.host_step, "f32"),
}

WORKLOAD_TEXT = {
    "t3_decode_f32": "BASELINE configs[1]: T3 batched decode step, 24 layers x (residual-add+"
                     "LayerNorm, GELU-tanh [256,4096], residual-add+LayerNorm), B=256, hidden "
                     "1024, f32",
    "t3_decode_bf16": "BASELINE configs[1], bf16 activations / f32 statistics variant",
    "t3_prefill_f32": "BASELINE configs[0]: T3 prefill layer-op stack f32, T=512",
    "t3_prefill_large_bf16": "BASELINE configs[2]: T3 large prefill B=64 x T=1024 (65536 rows), "
                             "hidden 1024, MLP 4096: embedding gather-add, residual-add+"
                             "LayerNorm and GELU-tanh on bf16, f32 stats",
    "t3_prefill_seq_f16": "T3 prefill input sequence [speaker ; prompt ; text] + positions, 64 "
                          "utterances x 1024 rows, f16 tables (text 50276x1024), f32 out",
    "cfm_ops_f32": "BASELINE configs[3]: CFM LN over C + Mish [32,256,1000] f32 + timestep "
                   "embedding",
    "cfm_act_f32": "SiLU and Mish standalone on [32,256,1000] f32",
    "cfm_block_tail_f32": "GEMM-epilogue neighbour: CFM conv bias + transpose + LN over C + "
                          "Mish + mask, [32,256,1000] -> [32,1000,256] f32",
    "hift_snake_f32": "BASELINE configs[4]: HiFT Snake B=16, 3 stages, f32",
    "hift_snake_btc_f32": "BASELINE configs[4] shapes in the engine's [B][T][C] layout",
    "t3_fc_epilogue_bf16": "GEMM-epilogue neighbour: T3 fc bias + GELU-tanh [65536, 4096] bf16",
    "s3gen_epilogue_f32": "GEMM-epilogue neighbours: CFM FF GELU-erf + HiFT ResBlock mean + LeakyReLU, f32",
    "hift_dsp_f32": "HiFT NSF source + STFT + iSTFT tail, 32 x 10 s, f32",
    "t3_decode_step_f32": "elementwise share of a batched T3 decode step with the "
                          "KV-cache append, B=256, 24 layers, f32",
}


def make_workload(name, torch, dev, seed, rank=0, world=1):
    """The workload on this rank: strong-scaled ones take their
    shard of the job, the others a full batch of their own."""
    if name not in WORKLOADS:
        raise SystemExit(f"unknown workload {name!r}: {sorted(WORKLOADS)}")
    ctor = WORKLOADS[name][0]
    if getattr(ctor, "strong", False):
        return ctor(torch, dev, seed, rank=rank, world=world)
    return ctor(torch, dev, seed)


def host_sample(name, budget_s):
    """Run the workload's host step on the oracle until `budget_s`; returns
    (bytes, seconds, description)."""
    fn, nb, _, desc = WORKLOADS[name][1]()
    fn()  # warm (page in, thread pool)
    done, t0 = 0, time.perf_counter()
    while True:
        fn()
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s or done >= 10_000:
            break
    return nb * done, el, f"{done} x {desc}"


# ---------------------------------------------------------------- timing --

def capture(torch, launches, L, warm=3):
    """Warm the launches up eagerly, then capture them into one CUDA graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            for l in launches:
                _check(l.fn(s.cuda_stream), L)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st = torch.cuda.current_stream().cuda_stream
        for l in launches:
            _check(l.fn(st), L)
    torch.cuda.synchronize()
    return g


def time_graph(torch, g, reps, warm):
    for _ in range(warm):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / 1e3


def kernel_roofline(torch, wl, L, peak, reps=200):
    """Mean launch time of each kernel group on the step's own buffers, as a
    graph of that group's launches (in step order, repeated to at least 16
    launches) replayed at least `reps` times."""
    groups = {}
    for l in wl.launches:
        groups.setdefault(l.group, []).append(l)
    res = {}
    for name, ls in groups.items():
        # at least 16 launches per graph, so graph-launch gaps do not count
        ls = ls * max(1, -(-16 // len(ls)))
        g = capture(torch, ls, L, warm=1)
        # at least `reps` replays, and enough for CBX_ROOFLINE_MIN_S (0.5 s) of
        # this group's kernels
        min_s = float(os.environ.get("CBX_ROOFLINE_MIN_S", "0.5"))
        t10 = time_graph(torch, g, 10, 3)
        n_reps = max(reps, min(20000, int(min_s / max(t10 / 10, 1e-7))))
        t = time_graph(torch, g, n_reps, 0)
        per_launch = t / (n_reps * len(ls))
        nbytes = ls[0].nbytes
        res[name] = {"launches_per_step": len(groups[name]), "bytes_per_launch": nbytes,
                     "us_per_launch": per_launch * 1e6,
                     "achieved_gbs": nbytes / per_launch / 1e9}
        del g
    return res


def gpu_numa_node(torch, dev):
    """NUMA node of the GPU's PCI function (None when the platform does not say)."""
    try:
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        return node if node >= 0 else None
    except Exception:
        return None


def node_cpus(node):
    """CPU ids of a NUMA node (from sysfs), or None."""
    try:
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        return cpus
    except Exception:
        return None


class HostBuffers:
    """Pinned host copies of the workload's per-step inputs and outputs,
    allocated and first touched by this process while it runs on the CPUs of
    the GPU's NUMA node, so the pages sit next to the GPU's PCIe root."""

    def __init__(self, torch, wl, dev):
        self.numa_node = gpu_numa_node(torch, dev)
        cpus = node_cpus(self.numa_node) if self.numa_node is not None else None
        old = os.sched_getaffinity(0)
        placed = False
        if cpus and cpus & old:
            os.sched_setaffinity(0, cpus & old)
            placed = True
        try:
            self.h_in = [[t.cpu().pin_memory() for t in ins] for ins, _, _ in wl.chunks]
            self.h_out = [[torch.empty(t.shape, dtype=t.dtype, pin_memory=True).fill_(0)
                           for t in outs] for _, outs, _ in wl.chunks]
        finally:
            os.sched_setaffinity(0, old)
        self.placement = (f"NUMA node {self.numa_node} (first touch on its CPUs)" if placed else
                          "default placement (the GPU reports no NUMA node)")


def e2e_run(torch, wl, L, steps, warm, hb, kernels=True):
    """End to end through the C ABI with host buffers: per chunk (layer),
    pinned H2D of its activations -> its launches -> D2H of its outputs, on
    three streams so copies overlap the kernels of neighbouring chunks; then,
    for a sharded job on several ranks, the result gather to rank 0 over NCCL.
    With kernels=False only the copies run: the per-rank copy ceiling of the
    same traffic.  Returns (seconds, h2d bytes, d2h bytes, op bytes) of this rank."""
    from chatterbox_amdvulkan_b200 import shard
    h_in, h_out = hb.h_in, hb.h_out
    s_in, s_c, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    n = len(wl.chunks)
    e_in = [torch.cuda.Event() for _ in range(n)]
    e_c = [torch.cuda.Event() for _ in range(n)]
    e_o = [torch.cuda.Event() for _ in range(n)]
    h2d = sum(t.numel() * t.element_size() for ins, _, _ in wl.chunks for t in ins)
    d2h = sum(t.numel() * t.element_size() for _, outs, _ in wl.chunks for t in outs)
    op_bytes = sum(l.nbytes for _, _, lz in wl.chunks for l in lz)
    gather = wl.gather if kernels and wl.gather is not None and shard.env_rank()[2] > 1 else None

    def step():
        for i, (ins, outs, lz) in enumerate(wl.chunks):
            with torch.cuda.stream(s_in):
                s_in.wait_event(e_c[i])          # previous step's kernels done with inputs
                for d, h in zip(ins, h_in[i]):
                    d.copy_(h, non_blocking=True)
                e_in[i].record(s_in)
            s_c.wait_event(e_in[i])
            s_c.wait_event(e_o[i])               # previous step's outputs copied out
            st = s_c.cuda_stream
            if kernels:
                for l in lz:
                    _check(l.fn(st), L)
            e_c[i].record(s_c)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e_c[i])
                for d, h in zip(outs, h_out[i]):
                    h.copy_(d, non_blocking=True)
                e_o[i].record(s_out)
        if gather is not None:
            with torch.cuda.stream(s_c):
                shard.gather_rows_into(*gather)

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    if shard.env_rank()[2] > 1:
        import torch.distributed as dist
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for _ in range(steps):
        step()
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_c)
    t1.record(s_out)
    t1.synchronize()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / 1e3, h2d, d2h, op_bytes


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ arms --

def run_reference(args):
    """CPU oracle on the host cores, same metric/config as ours; rank 0 only."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return 0
    import oracle as O
    O.build()
    cores = cpu_cores()
    O.set_threads(cores)
    fn, nb, rows, desc = WORKLOADS[args.workload][1]()
    t0 = time.perf_counter()
    fn()
    t_one = time.perf_counter() - t0
    # size the per-step sample so that warmup + steps end within the budget
    budget = float(os.environ.get("CBX_REF_BUDGET_S", "120"))
    reps = max(1, min(int(budget / max(t_one, 1e-6) / max(1, args.steps + args.warmup)), 1000))
    for _ in range(args.warmup):
        for _ in range(reps):
            fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(reps):
            fn()
    el = time.perf_counter() - t0
    per_step = el / args.steps
    value = nb * reps / per_step / 1e9
    sample = f"{reps} x {desc} per step"
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
            "higher_is_better": True,
            "scaling": ("strong" if getattr(WORKLOADS[args.workload][0], "strong", False)
                        else "weak"),
            "vs_baseline": None,
            "dtype": WORKLOADS[args.workload][2], "data": "synthetic (seeded)",
            "impl": "reference",
            "config": {"workload": WORKLOAD_TEXT[args.workload], "name": args.workload,
                       "sample_bytes_per_step": nb * reps},
            "rows_per_s": round(rows * reps / per_step, 1),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores,
                             "kind": "port", "sample": sample,
                             "note": "oracle/cbx_oracle.c: C restatement of the engine's ggml "
                                     "op composition (OpenMP, f64 transcendentals); ggml's CPU "
                                     "backend is an empty submodule in the reference checkout"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist

    from chatterbox_amdvulkan_b200 import _lib, shard

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (libcbx_ops has no CPU path)")
    rank, local, world = shard.init("nccl")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = _lib.load()
    peak, peak_kind = load_peaks()
    wl = make_workload(args.workload, torch, dev, seed=1000 + rank, rank=rank, world=world)
    bytes_step = wl.bytes_per_step
    # whole-job bytes and rows per step: the fixed job when it is sharded
    # (strong scaling), else every rank's own batch (weak scaling)
    job_bytes = wl.job_bytes_per_step if wl.strong else bytes_step * world
    job_rows = wl.job_rows if wl.strong else wl.rows * world
    sets = wl.all_sets
    # The timed steps run as few CUDA graphs as possible: one graph holds
    # `per_graph` consecutive steps (whole rotations of the input sets, at
    # most ~2048 launches, and all of `steps` when they fit), so the steps
    # chain by programmatic dependent launch with no graph-launch gap between
    # them; single-step graphs cover a remainder, so exactly `steps` steps are
    # timed either way.
    per_rot = len(wl.launches) * len(sets)        # launches per rotation of the sets
    max_rot = max(1, 2048 // per_rot)
    steps_rot = max(args.steps // len(sets), 1)   # whole rotations in the timed steps
    n_big = -(-steps_rot // max_rot)               # graphs of equal size that cover them
    rots = max(1, steps_rot // n_big)
    per_graph = rots * len(sets)
    big = capture(torch, [l for _ in range(rots) for lz in sets for l in lz], L)
    graphs = [capture(torch, lz, L) for lz in sets]

    def run_steps(n):
        for _ in range(n // per_graph):
            big.replay()
        for k in range(n % per_graph):
            graphs[k % len(graphs)].replay()

    run_steps(args.warmup)
    # every graph the timed region replays has run once before it (untimed)
    big.replay()
    for g_ in graphs:
        g_.replay()
    torch.cuda.synchronize()

    gpu_id = None
    try:
        props = torch.cuda.get_device_properties(dev)
        gpu_id = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    except Exception:
        pass
    sampler = ClockSampler(gpu_id)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run_steps(args.steps)
    e1.record()
    e1.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t_local = e0.elapsed_time(e1) / 1e3
    t = shard.max_over_ranks(t_local)
    per_step = t / args.steps
    value = job_bytes / per_step / 1e9
    rows_s = job_rows / per_step

    # dominant kernel: mean launch time per kernel group on the step's buffers
    class _All:
        launches = [l for lz in sets for l in lz]
    rsampler = ClockSampler(gpu_id)
    rsampler.start()
    kr = kernel_roofline(torch, _All, L, peak,
                         reps=int(os.environ.get("CBX_ROOFLINE_REPS", "200")))
    rclocks = rsampler.stop()
    for v in kr.values():
        v["launches_per_step"] //= len(sets)
    dom = max(kr, key=lambda k: kr[k]["us_per_launch"] * kr[k]["launches_per_step"])
    traffic = load_traffic().get(f"{wl.name}:{dom}", {}).get("bytes_per_launch")
    if traffic is not None and wl.strong:
        # the committed capture is of the whole job on one GPU: scale to this shard
        traffic = int(traffic * wl.rows / wl.job_rows)
    roof = {"bound": "hbm", "kernel": dom, "achieved": round(kr[dom]["achieved_gbs"], 1),
            "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(kr[dom]["achieved_gbs"] / peak, 4),
            "traffic": traffic, "algorithmic_bytes_per_launch": kr[dom]["bytes_per_launch"],
            "us_per_launch": round(kr[dom]["us_per_launch"], 3),
            "clocks": rclocks,
            "per_kernel": {k: {kk: (round(vv, 3) if isinstance(vv, float) else vv)
                               for kk, vv in v.items()} for k, v in kr.items()}}

    # end to end through the C ABI with host buffers
    e2e = None
    if not args.no_e2e:
        e2e_steps = max(3, min(args.steps, args.e2e_steps))
        hb = HostBuffers(torch, wl, dev)
        te, h2d, d2h, op_bytes = e2e_run(torch, wl, L, e2e_steps, 2, hb)
        te = shard.max_over_ranks(te)
        # the same copies without kernels or gather: this rank's copy ceiling
        tc, _, _, _ = e2e_run(torch, wl, L, e2e_steps, 2, hb, kernels=False)
        tc = shard.max_over_ranks(tc)
        # one pass over the chunks covers op_bytes / bytes_step workload steps
        # (several with rotating input sets)
        eq = op_bytes / bytes_step
        t_step = te / (e2e_steps * eq)
        c_step = tc / (e2e_steps * eq)
        e2e_value = job_bytes / t_step / 1e9
        ceil_value = job_bytes / c_step / 1e9
        e2e = {"value": round(e2e_value, 3), "unit": "GB/s",
               "h2d_bytes_per_step": int(h2d / eq), "d2h_bytes_per_step": int(d2h / eq),
               "steps": int(round(e2e_steps * eq)), "ms_per_step": round(t_step * 1e3, 4),
               "how": ("pinned host buffers on each rank; per chunk H2D -> kernels -> D2H on 3 "
                       "streams" + ("; then the result rows gathered to rank 0 over NCCL"
                                    if world > 1 and wl.gather is not None else "")),
               "host_memory": hb.placement,
               "copy_ceiling": {"value": round(ceil_value, 3), "unit": "GB/s",
                                "ms_per_step": round(c_step * 1e3, 4),
                                "h2d_gbs_per_rank": round(h2d / eq / c_step / 1e9, 2),
                                "d2h_gbs_per_rank": round(d2h / eq / c_step / 1e9, 2),
                                "how": "the same pinned copies on the same streams, no kernels "
                                       "or gather, all ranks at once (max over ranks)"},
               "frac_of_copy_ceiling": round(e2e_value / ceil_value, 4)}
        if world > 1 and wl.gather is not None:
            y, _, counts = wl.gather
            e2e["gather"] = {"rows": sum(counts), "bytes_to_rank0": sum(counts[1:]) * (
                y.numel() // max(1, y.shape[0])) * y.element_size(), "backend": "nccl send/recv"}
        del hb

    # final result gather over NCCL, timed alone (the e2e number includes it)
    gather = None
    if world > 1:
        if wl.gather is not None:
            def do_gather():
                shard.gather_rows_into(*wl.gather)
            g_bytes = wl.gather[0].numel() * wl.gather[0].element_size()
        else:
            last = wl.chunks[-1][1][0]

            def do_gather():
                shard.gather_rows(last.view(1, -1), counts=[1] * world)
            g_bytes = last.numel() * last.element_size()
        do_gather()  # first call sets up the NCCL channels
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        do_gather()
        g1.record()
        g1.synchronize()
        gather = {"ms": round(shard.max_over_ranks(g0.elapsed_time(g1)), 4),
                  "bytes_per_rank": g_bytes, "backend": "nccl send/recv to rank 0"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O
        O.build()
        cores = cpu_cores()
        O.set_threads(cores)
        nb, el, desc = host_sample(args.workload, float(os.environ.get("CBX_CPU_BUDGET_S", "15")))
        cpu = {"value": round(nb / el / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": desc + f" in {el:.2f} s"}
        # the same port on one thread, for context
        O.set_threads(1)
        nb1, el1, desc1 = host_sample(args.workload,
                                      float(os.environ.get("CBX_CPU_BUDGET_1T_S", "4")))
        O.set_threads(cores)
        cpu["single_thread"] = {"value": round(nb1 / el1 / 1e9, 3), "unit": "GB/s", "cores": 1,
                                "sample": desc1 + f" in {el1:.2f} s"}

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
                "higher_is_better": True, "scaling": "strong" if wl.strong else "weak",
                "vs_baseline": None, "dtype": wl.dtype,
                "data": ("synthetic (seeded N(0,1) with 1% +-20 outliers)"
                         if wl.name.startswith("t3_decode") else "synthetic (seeded)"),
                "config": {"workload": wl.workload, "name": wl.name,
                           "rows_per_gpu": wl.rows, "global_rows": job_rows,
                           "bytes_per_step_per_gpu": bytes_step,
                           "bytes_per_step_job": job_bytes,
                           "l2": (f"inputs larger than L2 ({bytes_step / 1e6:.0f} MB per step "
                                  "per GPU, every op on its own buffers)" if len(sets) == 1 else
                                  f"inputs larger than L2: {len(sets)} rotating input sets "
                                  f"({bytes_step * len(sets) / 1e6:.0f} MB)"),
                           "parallelism": (f"dp{world}: the job's {job_rows} rows split into "
                                           f"{world} contiguous shards, no collective in the "
                                           "timed region" if wl.strong else
                                           f"dp{world} (independent rows per GPU, no collective"
                                           " in the timed region)"),
                           "launch": f"CUDA graphs of {per_graph} step(s) x {len(wl.launches)} "
                                     "launches, "
                                     + ("programmatic dependent launch"
                                        if os.environ.get("CBX_DISABLE_PDL", "0") in ("", "0")
                                        else "plain launches"),
                           **({"gather_entry_point": wl.gather_call}
                              if getattr(wl, "gather_call", None) else {})},
                "rows_per_s": round(rows_s, 1),
                "frac_of_peak_per_gpu": round(value / world / peak, 4),
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": len(wl.launches) * args.steps, "clocks": clocks}
        if gather:
            line["gather"] = gather
        print(json.dumps(line), flush=True)
    del graphs, big
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="t3_prefill_large_bf16",
                    help="t3_prefill_large_bf16 (default, configs[2], sharded across ranks), "
                         "t3_decode_f32 (configs[1]), t3_decode_bf16, t3_prefill_f32 "
                         "(configs[0]), t3_prefill_seq_f16 (the T3 prefill input sequence with "
                         "the 50276-row text table), cfm_ops_f32 "
                         "(configs[3]), cfm_act_f32 (standalone SiLU / Mish), hift_snake_f32 (configs[4]), hift_snake_btc_f32, "
                         "t3_fc_epilogue_bf16, s3gen_epilogue_f32, cfm_block_tail_f32 "
                         "(GEMM-epilogue neighbours), t3_decode_step_f32 "
                         "(batched decode step with the KV-cache append), hift_dsp_f32 (HiFT NSF "
                         "source, STFT, iSTFT tail)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
