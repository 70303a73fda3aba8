"""Seeded randomized sweep of the C ABI against the oracle: many small random
shapes, dtypes, row strides, misaligned base pointers and in-place calls per
entry point (the hand-picked cases in the other GPU tests cover the configured
shapes; this one covers the space between them).  Same bars as the parity
tests: bit-exact for gathers, sums and copies; 1e-6 + 1e-5 |ref| for f32;
2 ulp for 16-bit outputs."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from _gpu import TORCH_OF, dev, host, host_f32
from conftest import assert_close_f32, assert_within_bf16_ulps

pytestmark = pytest.mark.gpu

TYPES = [O.F32, O.BF16, O.F16]


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


def _close(got, ref, t, what):
    if t == O.F32:
        assert_close_f32(got, ref, what=what)
    elif t == O.BF16:
        assert_within_bf16_ulps(got, ref, ulps=2, what=what)
    else:
        r16 = np.asarray(ref, np.float32).astype(np.float16).astype(np.float64)
        fin = np.isfinite(r16)
        ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(r16[fin]), 2.0 ** -14))) - 10)
        assert np.all(np.abs(np.asarray(got, np.float64)[fin] - r16[fin]) <= 2 * ulp), what


def _offset_view(a, t, off):
    """Device copy of oracle-storage array `a` starting `off` elements into a
    larger buffer (off > 0: a base pointer that is not 16-byte aligned)."""
    flat = dev(np.ascontiguousarray(a).reshape(-1), t)
    buf = torch.zeros(flat.numel() + off, dtype=flat.dtype, device="cuda")
    buf[off:] = flat
    return buf[off:].view(a.shape)


@pytest.mark.parametrize("seed", range(12))
def test_sweep_add_layernorm(ops, seed):
    rng = np.random.default_rng(1000 + seed)
    t = TYPES[seed % 3]
    H = int(rng.choice([1, 7, 32, 100, 256, 333, 1024, 1536, 2048, 4100]))
    N = int(rng.integers(1, 700))
    off = int(rng.choice([0, 0, 1, 3]))
    x = (rng.standard_normal((N, H)) * rng.uniform(0.5, 4) + rng.uniform(-1, 1)).astype(np.float32)
    r = rng.standard_normal((N, H)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    b = (0.1 * rng.standard_normal(H)).astype(np.float32)
    xq, rq = O.to_type(x, t), O.to_type(r, t)
    s_ref, y_ref = O.add_layernorm(xq, rq, g, b, 1e-5, in_t=t, out_t=O.F32)
    xd, rd = _offset_view(xq, t, off), _offset_view(rq, t, off)
    y, s = ops.add_layernorm(xd, rd, dev(g), dev(b), 1e-5, out_dtype=torch.float32,
                             return_sum=True)
    assert np.array_equal(host(s), s_ref), f"sum exact H={H} N={N} t={t} off={off}"
    assert_close_f32(host(y), y_ref, what=f"ln H={H} N={N} t={t} off={off}")


@pytest.mark.parametrize("seed", range(12))
def test_sweep_unary_and_bias_act(ops, seed):
    rng = np.random.default_rng(2000 + seed)
    t = TYPES[seed % 3]
    H = int(rng.choice([1, 3, 8, 64, 250, 1024, 4096]))
    N = int(rng.integers(1, 300))
    off = int(rng.choice([0, 1, 2]))
    x = (3 * rng.standard_normal((N, H))).astype(np.float32)
    x.reshape(-1)[: min(8, x.size)] = [0, -0.0, 20, -20, 19.99, 25, -25, 1e-6][: min(8, x.size)]
    xq = O.to_type(x, t)
    xf = O.to_f32(xq, t)
    name, fn, ref = [("gelu", ops.gelu, O.gelu_tanh), ("silu", ops.silu, O.silu),
                     ("mish", ops.mish, O.mish), ("gelu_erf", ops.gelu_erf, O.gelu_erf)][seed % 4]
    got = fn(_offset_view(xq, t, off))
    _close(host_f32(got), ref(xf), t, f"{name} N={N} H={H} t={t} off={off}")
    # bias + activation along ne0 / ne1
    act = ["gelu", "leaky_relu", "elu", None][seed % 4]
    code = {"gelu": O.ACT_GELU, "leaky_relu": O.ACT_LEAKY_RELU, "elu": O.ACT_ELU, None: O.ACT_NONE}
    axis = "ne0" if seed % 2 == 0 else "ne1"
    blen = H if axis == "ne0" else int(rng.integers(1, 9))
    bias = rng.standard_normal(blen).astype(np.float32)
    got = ops.bias_act(_offset_view(xq, t, off), dev(bias), act, axis=axis, act_param=0.2)
    ref = O.bias_act(xf, bias, O.BIAS_NE0 if axis == "ne0" else O.BIAS_NE1, code[act], 0.2,
                     bias_len=blen)
    _close(host_f32(got), ref, t, f"bias_act {act} {axis} N={N} H={H} t={t} off={off}")


@pytest.mark.parametrize("seed", range(8))
def test_sweep_embed_and_sum3_bit_exact(ops, seed):
    rng = np.random.default_rng(3000 + seed)
    t = TYPES[seed % 3]
    V, P = int(rng.integers(1, 300)), int(rng.integers(1, 200))
    H = int(rng.choice([1, 5, 64, 96, 1024]))
    n = int(rng.integers(1, 400))
    tok = O.to_type((0.02 * rng.standard_normal((V, H))).astype(np.float32), t)
    pos = O.to_type((0.02 * rng.standard_normal((P, H))).astype(np.float32), t)
    ids = rng.integers(-2, V + 2, n).astype(np.int32)          # includes out-of-range ids
    off = int(rng.integers(0, P + 3))
    ref, rerr = O.embed_gather_add(tok, t, ids, pos, t, pos_offset=off, out_t=t)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = ops.embed_gather_add(dev(tok, t), torch.from_numpy(ids).cuda(), dev(pos, t),
                               n_past=off, out_dtype=TORCH_OF[t], err_word=err)
    assert int(host(err)[0]) == rerr
    assert np.array_equal(host(got), ref), f"embed V={V} P={P} H={H} n={n} t={t}"
    m = int(rng.integers(1, 5000))
    a, b, c = (O.to_type(rng.standard_normal(m).astype(np.float32), t) for _ in range(3))
    s = np.float32(rng.uniform(0.1, 1))
    got = ops.sum3_scale(dev(a, t), dev(b, t), dev(c, t), float(s))
    assert np.array_equal(host(got), O.sum3_scale(a, b, c, s, t)), f"sum3 m={m} t={t}"


@pytest.mark.parametrize("seed", range(8))
def test_sweep_layernorm_channels_and_snake(ops, seed):
    rng = np.random.default_rng(4000 + seed)
    B = int(rng.integers(1, 4))
    C = int(rng.choice([8, 32, 64, 100, 128, 256]))
    T = int(rng.choice([1, 3, 16, 37, 64, 129, 1000]))
    x = (2 * rng.standard_normal((B, C, T)) + 0.3).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    mask = (rng.random((B, T)) > 0.2).astype(np.float32) if seed % 2 else None
    layout = "BCT" if seed % 3 else "BTC"
    xl = x if layout == "BCT" else np.ascontiguousarray(x.transpose(0, 2, 1))
    act = "mish" if seed % 2 == 0 else None
    got = ops.layernorm_channels(dev(xl), dev(g), dev(b), 1e-5,
                                 None if mask is None else dev(mask), layout=layout, act=act)
    ref = O.layernorm_channels(xl, g, b, 1e-5, mask, O.BCT if layout == "BCT" else O.BTC,
                               O.ACT_MISH if act else O.ACT_NONE)
    assert_close_f32(host(got), ref, what=f"ln_C B={B} C={C} T={T} {layout} mask={mask is not None}")
    alpha = np.exp(0.3 * rng.standard_normal(C)).astype(np.float32)
    got = ops.snake(dev(xl), dev(alpha), layout=layout)
    ref = O.snake(xl, alpha, layout=O.BCT if layout == "BCT" else O.BTC)
    assert_close_f32(host(got), ref, what=f"snake B={B} C={C} T={T} {layout}")


@pytest.mark.parametrize("seed", range(10))
def test_sweep_causal_block1d_tail(ops, seed):
    """Random shapes around the TMA kernel's conditions (C in {32..256},
    T % 4, T >= 16, 16-byte aligned x and y) and the per-column fallback."""
    rng = np.random.default_rng(5000 + seed)
    B = int(rng.integers(1, 5))
    C = int(rng.choice([32, 64, 128, 256, 80, 100, 512]))
    T = int(rng.choice([1, 5, 15, 16, 17, 20, 33, 64, 100, 257, 1000]))
    off = int(rng.choice([0, 0, 0, 1]))
    x = (2 * rng.standard_normal((B, C, T)) + rng.uniform(-1, 1)).astype(np.float32)
    cb = (0.5 * rng.standard_normal(C)).astype(np.float32) if seed % 3 else None
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32) if seed % 2 else None
    mask = (rng.random((B, T)) > 0.3).astype(np.float32) if seed % 4 else None
    act = [O.ACT_MISH, O.ACT_NONE, O.ACT_SILU][seed % 3]
    ref = O.causal_block1d_tail(x, cb, g, b, 1e-5, mask, act)
    got = ops.causal_block1d_tail(_offset_view(x, O.F32, off), None if cb is None else dev(cb),
                                  dev(g), None if b is None else dev(b), 1e-5,
                                  None if mask is None else dev(mask),
                                  {O.ACT_MISH: "mish", O.ACT_NONE: None, O.ACT_SILU: "silu"}[act])
    assert_close_f32(host(got), ref, what=f"tail B={B} C={C} T={T} off={off} act={act}")


@pytest.mark.parametrize("seed", range(10))
def test_sweep_stft_istft(ops, seed):
    """Random lengths, batches, layouts and offsets for the engine's sizes
    (persistent bulk-copy kernels when aligned) and n_fft 8 / hop 2."""
    rng = np.random.default_rng(6000 + seed)
    n_fft, hop = [(16, 4), (8, 2)][seed % 2]
    B = int(rng.integers(1, 6))
    layout = "BTC" if seed % 3 else "BCT"
    lay = O.BTC if layout == "BTC" else O.BCT
    off = int(rng.choice([0, 0, 1, 2]))
    win = O.hann_window(n_fft)
    T = int(rng.integers(n_fft // 2 + 1, 5000))
    x = (0.3 * rng.standard_normal((B, T))).astype(np.float32)
    got = ops.stft(_offset_view(x, O.F32, off), n_fft, hop, dev(win), layout=layout)
    assert_close_f32(host(got), O.stft(x, n_fft, hop, win, layout=lay),
                     what=f"stft {n_fft}/{hop} B={B} T={T} {layout} off={off}")
    Tf = int(rng.integers(2, 1500))
    nb = n_fft // 2 + 1
    p = np.concatenate([rng.normal(-2.0, 0.9, (B, nb, Tf)), rng.normal(0.0, 3.0, (B, nb, Tf))],
                       axis=1).astype(np.float32)
    pl = np.ascontiguousarray(p.transpose(0, 2, 1)) if layout == "BTC" else p
    got = ops.istft_post(_offset_view(pl, O.F32, off), n_fft, hop, dev(win), layout=layout,
                         audio_limit=np.inf)
    assert_close_f32(host(got), O.istft_post(pl, n_fft, hop, win, layout=lay, audio_limit=np.inf),
                     what=f"istft {n_fft}/{hop} B={B} Tf={Tf} {layout} off={off}")


@pytest.mark.parametrize("seed", range(6))
def test_sweep_nsf_source(ops, seed):
    """Random batch, length, upsample (both frame-start paths) and rate."""
    rng = np.random.default_rng(7000 + seed)
    B = int(rng.integers(1, 5))
    n_mel = int(rng.integers(1, 120))
    up = int(rng.choice([18, 20, 64, 99, 256, 480]))
    sr = int(rng.choice([16000, 22050, 24000]))
    f0 = np.where(rng.random((B, n_mel)) < 0.25, 0.0,
                  rng.uniform(60, 420, (B, n_mel))).astype(np.float32)
    phase = rng.uniform(-np.pi, np.pi, (B, 9)).astype(np.float32)
    noise = rng.standard_normal((B, 9, n_mel * up)).astype(np.float32)
    lw = (0.4 * rng.standard_normal(9)).astype(np.float32)
    lb = float(rng.uniform(-0.05, 0.05))
    got = ops.nsf_source(dev(f0), up, dev(phase), dev(noise), lw, lb, sr)
    ref = O.nsf_source(f0, up, phase, noise, lw, lb, sampling_rate=sr)
    assert_close_f32(host(got), ref, what=f"nsf B={B} n_mel={n_mel} up={up} sr={sr}")
