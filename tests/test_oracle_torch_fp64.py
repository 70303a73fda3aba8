"""Cross-check of the CPU oracle against torch CPU float64 on the formulas it
restates (LayerNorm with biased variance, GELU-tanh, SiLU, Mish with the
softplus threshold, exact GELU, LN over C in [B,C,T], Snake, the sinusoid):
the oracle's f32 results equal the float64 results rounded once to f32 within
1 ulp, except where the engine's node-by-node f32 roundings are the
specification (Snake's five nodes, the LN affine), which are checked at the
f32 parity bar.  CPU only."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from conftest import assert_close_f32


def _ulps(got, ref64):
    ref32 = ref64.astype(np.float32)
    a = np.abs(ref32.astype(np.float64))
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -126))) - 23)
    return np.abs(got.astype(np.float64) - ref32.astype(np.float64)) / ulp


@pytest.fixture(scope="module")
def x():
    rng = np.random.default_rng(11)
    v = (3.0 * rng.standard_normal(20000)).astype(np.float32)
    v[:8] = [0.0, -0.0, 19.99, 20.0, 20.01, -20.0, 25.0, -25.0]
    return v


def test_activations_match_fp64(x):
    t = torch.from_numpy(x).double()
    u = np.sqrt(2 / np.pi) * (t + 0.044715 * t ** 3)
    gelu = t * torch.sigmoid(2.0 * u)          # = 0.5 t (1 + tanh u), without cancellation
    assert _ulps(O.gelu_tanh(x), gelu.numpy()).max() <= 1.0
    assert _ulps(O.silu(x), (t * torch.sigmoid(t)).numpy()).max() <= 1.0
    sp = torch.where(t > 20, t, torch.log1p(torch.exp(t)))
    # Mish is three ggml nodes, each rounded to f32 (softplus, tanh, mul)
    assert _ulps(O.mish(x), (t * torch.tanh(sp)).numpy()).max() <= 3.0
    gerf = 0.5 * t * torch.special.erfc(-t / np.sqrt(2.0))
    assert _ulps(O.gelu_erf(x), gerf.numpy()).max() <= 1.0


def test_layernorm_matches_fp64():
    rng = np.random.default_rng(12)
    xs = rng.standard_normal((64, 1024)).astype(np.float32) * 2 + 0.3
    r = rng.standard_normal((64, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    s, y = O.add_layernorm(xs, r, g, b, 1e-5)
    s64 = torch.from_numpy(xs).double() + torch.from_numpy(r).double()
    assert np.array_equal(s, s64.float().numpy())     # the residual sum is one IEEE add
    ref = torch.nn.functional.layer_norm(torch.from_numpy(s).double(), (1024,),
                                         torch.from_numpy(g).double(),
                                         torch.from_numpy(b).double(), 1e-5)
    assert_close_f32(y, ref.float().numpy(), what="ln vs fp64")


def test_layernorm_channels_matches_fp64():
    rng = np.random.default_rng(13)
    xs = rng.standard_normal((2, 256, 37)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    b = (0.1 * rng.standard_normal(256)).astype(np.float32)
    y = O.layernorm_channels(xs, g, b, 1e-5, None, O.BCT, O.ACT_NONE)
    t = torch.from_numpy(xs).double().transpose(1, 2)
    ref = torch.nn.functional.layer_norm(t, (256,), torch.from_numpy(g).double(),
                                         torch.from_numpy(b).double(), 1e-5).transpose(1, 2)
    assert_close_f32(y, ref.float().numpy(), what="ln over C vs fp64")


def test_snake_and_sinusoid_match_fp64():
    rng = np.random.default_rng(14)
    xs = rng.standard_normal((1, 8, 500)).astype(np.float32)
    a = np.exp(0.3 * rng.standard_normal(8)).astype(np.float32)
    t, ta = torch.from_numpy(xs).double(), torch.from_numpy(a).double()[None, :, None]
    ref = t + torch.sin(t * ta) ** 2 / (ta + 1e-9)
    assert_close_f32(O.snake(xs, a), ref.float().numpy(), what="snake vs fp64")
    ts = rng.random(16).astype(np.float32)
    fr = torch.from_numpy(O.sinusoid_freqs(320)).double()
    arg = (1000.0 * torch.from_numpy(ts).double())[:, None] * fr[None, :]
    emb = torch.cat([torch.sin(arg), torch.cos(arg)], dim=1).numpy()
    # |a| up to 1000 rad: the f32 argument's rounding (<= 2 ulp of a) dominates
    got = O.timestep_embed(ts, 320, 1000.0)
    a32 = (np.float32(1000.0) * ts)[:, None].astype(np.float32) * np.concatenate(
        [O.sinusoid_freqs(320)] * 2)[None, :]
    ulp_a = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(a32), 2.0 ** -126))) - 23)
    assert np.all(np.abs(got - emb) <= 1e-6 + 1e-5 * np.abs(emb) + 2.0 * ulp_a)
