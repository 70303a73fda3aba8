"""GPU parity: every libcbx_ops entry point (called through the C ABI) against
the CPU oracle on the same seeded inputs.

Bars (from the build's contract): gathers bit-exact; f32 ops
|gpu - ref| <= 1e-6 + 1e-5 |ref|; bf16 outputs within 2 bf16 ulp of the
oracle's f32 result rounded to bf16 (f16 outputs: 2 f16 ulp)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from _gpu import dev, host, host_f32, normal_with_outliers
from conftest import assert_close_f32, assert_within_bf16_ulps

pytestmark = pytest.mark.gpu

EPS = 1e-5


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


def _f16_close(got_f32, ref_f32, ulps=2):
    ref16 = np.asarray(ref_f32, np.float32).astype(np.float16).astype(np.float64)
    got = np.asarray(got_f32, np.float64)
    fin = np.isfinite(ref16)
    a = np.abs(ref16[fin])
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -14))) - 10)
    assert np.all(np.abs(got[fin] - ref16[fin]) <= ulps * ulp)


def _check_typed(got_t, ref_f32, t, what):
    if t == O.F32:
        assert_close_f32(host(got_t), ref_f32, what=what)
    elif t == O.BF16:
        assert_within_bf16_ulps(host_f32(got_t), ref_f32, what=what)
    else:
        _f16_close(host_f32(got_t), ref_f32)


# ------------------------------------------------------------ golden pins --

def test_gpu_matches_reference_goldens(ops, golden):
    """The GPU path against the reference NumPy oracle outputs directly."""
    g = golden
    assert_close_f32(host(ops.gelu(dev(g["gelu_x"]))), g["gelu_y"], what="gelu")
    y, s = ops.add_layernorm(dev(g["ln_x"]), dev(g["ln_r"]), dev(g["ln_w"]), dev(g["ln_b"]),
                             EPS, return_sum=True)
    assert np.array_equal(host(s), g["ln_s"])
    assert_close_f32(host(y), g["ln_y"], what="ln")
    assert_close_f32(host(ops.layer_norm(dev(g["ln2_x"]), dev(g["ln2_w"]), dev(g["ln2_b"]))),
                     g["ln2_y"], what="ln ragged")
    assert_close_f32(host(ops.silu(dev(g["act_x"]))), g["silu_y"], what="silu")
    assert_close_f32(host(ops.mish(dev(g["act_x"]))), g["mish_y"], what="mish")
    y = ops.layernorm_channels(dev(g["cfm_x"]), dev(g["cfm_w"]), dev(g["cfm_b"]), EPS,
                               dev(g["cfm_mask"]), "BCT", "mish")
    assert_close_f32(host(y), g["cfm_y"], what="cfm")
    y = ops.causal_block1d_tail(dev(g["cbt_x"]), dev(g["cbt_cb"]), dev(g["cbt_w"]),
                                dev(g["cbt_b"]), EPS, dev(g["cbt_mask"]))
    assert_close_f32(host(y), g["cbt_y"], what="causal block tail")
    y = ops.snake(dev(g["snake_x"]), dev(g["snake_alpha"]))
    assert_close_f32(host(y), g["snake_y"], what="snake")
    y = ops.sinusoidal_pos_emb(dev(g["sin_t"]), 320, 1.0)
    assert_close_f32(host(y), g["sin_y_scale1"], what="sinusoid scale 1")
    n_past = int(g["emb_npast"][0])
    ids = torch.from_numpy(g["emb_ids"]).cuda()
    out = ops.embed_gather_add(dev(g["emb_tok"]), ids, dev(g["emb_pos"]), n_past=n_past)
    assert np.array_equal(host(out), g["emb_y"])
    out = ops.embed_gather_add(dev(g["emb_tok16"], O.F16), ids, dev(g["emb_pos16"], O.F16),
                               n_past=n_past)
    assert np.array_equal(host(out), g["emb16_y"])


# ------------------------------------------------------------ activations --

@pytest.mark.parametrize("t", [O.F32, O.BF16, O.F16])
@pytest.mark.parametrize("name", ["gelu", "silu", "mish"])
def test_activation_parity(ops, name, t):
    rng = np.random.default_rng(11)
    x32 = normal_with_outliers(rng, (4099,), frac=0.02) * 3.0   # ragged length
    x32[:6] = [0.0, -0.0, 20.0, -20.0, 25.0, -40.0]
    xq = O.to_type(x32, t)
    ref = getattr(O, {"gelu": "gelu_tanh"}.get(name, name))(O.to_f32(xq, t), O.F32)
    got = getattr(ops, name)(dev(xq, t))
    _check_typed(got, ref, t, f"{name} {t}")


@pytest.mark.parametrize("name", ["gelu", "silu", "mish"])
def test_activation_inplace_and_misaligned(ops, name):
    rng = np.random.default_rng(12)
    x = rng.standard_normal(10_001).astype(np.float32) * 4
    ref = getattr(O, {"gelu": "gelu_tanh"}.get(name, name))(x)
    xt = dev(x)
    getattr(ops, name)(xt, out=xt)                      # in place
    assert_close_f32(host(xt), ref, what="in place")
    buf = dev(np.concatenate([[0.0], x]).astype(np.float32))
    sub = buf[1:]                                        # 4-byte offset: scalar path
    got = getattr(ops, name)(sub)
    assert_close_f32(host(got), ref, what="misaligned")


def test_activation_special_values(ops):
    x = np.array([np.nan, np.inf, -np.inf, 88.0, -88.0, 1e30, -1e30, 1e-30], np.float32)
    for name, fn in (("gelu", O.gelu_tanh), ("silu", O.silu), ("mish", O.mish)):
        assert_close_f32(host(getattr(ops, name)(dev(x))), fn(x), what=name)


def test_gelu_config1_shape(ops):
    """Config 1's GELU input: [256, 4096] N(0,1) with 1% +-20 outliers."""
    rng = np.random.default_rng(1)
    x = normal_with_outliers(rng, (256, 4096))
    assert_close_f32(host(ops.gelu(dev(x))), O.gelu_tanh(x), what="gelu cfg1")


# --------------------------------------------------------------- layernorm --

@pytest.mark.parametrize("in_t,out_t", [(O.F32, O.F32), (O.BF16, O.BF16), (O.F32, O.BF16),
                                        (O.BF16, O.F32), (O.F16, O.F16)])
# paths: CTA per row (rows <= 4 x SMs, hidden/V a multiple of 32: 256x1024,
# 7x1024, 33x256, 2x4096); warp per row with affine prefetch (1000x1024);
# warp per row (5000x256, 5x320, 1x8192 -> generic; 8192x1024: more rows than
# resident warps, the balanced grid); generic (3x333).
@pytest.mark.parametrize("n_rows,H", [(256, 1024), (7, 1024), (33, 256), (5, 320), (3, 333),
                                      (2, 4096), (1, 8192), (1000, 1024), (5000, 256),
                                      (8192, 1024)])
def test_add_layernorm_parity(ops, in_t, out_t, n_rows, H):
    rng = np.random.default_rng(n_rows * 7 + H)
    x = O.to_type(normal_with_outliers(rng, (n_rows, H)), in_t)
    r = O.to_type(normal_with_outliers(rng, (n_rows, H)), in_t)
    g = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    b = (0.1 * rng.standard_normal(H)).astype(np.float32)
    s_ref, y_ref = O.add_layernorm(x, r, g, b, EPS, in_t=in_t, out_t=O.F32)
    y, s = ops.add_layernorm(dev(x, in_t), dev(r, in_t), dev(g), dev(b), EPS,
                             out_dtype={O.F32: torch.float32, O.BF16: torch.bfloat16,
                                        O.F16: torch.float16}[out_t], return_sum=True)
    assert np.array_equal(host(s), s_ref), "residual sum must be bit-exact"
    _check_typed(y, y_ref, out_t, f"ln {in_t}->{out_t} {n_rows}x{H}")


def test_layernorm_without_affine_or_residual(ops):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 1024)).astype(np.float32) * 5 + 3
    _, ref = O.add_layernorm(x, None, None, None, EPS)
    assert_close_f32(host(ops.layer_norm(dev(x), None, None)), ref)


def test_layernorm_in_place_and_strided(ops):
    """y == x in place, and a strided view (ggml nb[1] > ne0 * size)."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((16, 1024)).astype(np.float32)
    r = rng.standard_normal((16, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    s_ref, y_ref = O.add_layernorm(x, r, g, b, EPS)
    xt, rt = dev(x), dev(r)
    ops.add_layernorm(xt, rt, dev(g), dev(b), EPS, out=xt, return_sum=True, sum_out=rt)
    assert_close_f32(host(xt), y_ref, what="in place y")
    assert np.array_equal(host(rt), s_ref)
    # strided rows through the raw C ABI: rows of 1024 inside rows of 1536
    import ctypes
    from chatterbox_amdvulkan_b200 import _lib
    big = torch.zeros((16, 1536), device="cuda")
    big[:, :1024] = dev(x)
    yb = torch.full((16, 1536), 7.0, device="cuda")
    gt, bt = dev(g), dev(b)          # keep the tensors alive across the launch
    _lib.call("cbx_add_layernorm", ctypes.c_void_p(big.data_ptr()), None, O.F32, 1536,
              ctypes.c_void_p(gt.data_ptr()), ctypes.c_void_p(bt.data_ptr()),
              EPS, 16, 1024, None, ctypes.c_void_p(yb.data_ptr()), O.F32, 1536,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    _, y2 = O.add_layernorm(x, None, g, b, EPS)
    assert_close_f32(host(yb[:, :1024]), y2, what="strided")
    assert torch.all(yb[:, 1024:] == 7.0), "padding columns must be untouched"


def test_layernorm_config2_sampled_rows(ops):
    """Config 2 at full size: [65536, 1024] bf16 in/out, f32 stats; 2048 rows checked."""
    rng = np.random.default_rng(2)
    n, H = 65536, 1024
    xt = torch.randn((n, H), device="cuda", dtype=torch.float32).to(torch.bfloat16)
    rt = torch.randn((n, H), device="cuda", dtype=torch.float32).to(torch.bfloat16)
    g = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    b = (0.1 * rng.standard_normal(H)).astype(np.float32)
    y, s = ops.add_layernorm(xt, rt, dev(g), dev(b), EPS, return_sum=True)
    rows = np.sort(rng.choice(n, 2048, replace=False))
    xs, rs = host(xt[rows]), host(rt[rows])
    s_ref, y_ref = O.add_layernorm(xs, rs, g, b, EPS, in_t=O.BF16, out_t=O.F32)
    assert np.array_equal(host(s[rows]), s_ref)
    assert_within_bf16_ulps(host_f32(y[rows]), y_ref, what="cfg2 ln")


# ------------------------------------------------------ LN over channels --

# TMA path: T % 4 == 0, T >= 32, C <= 256, C % 8 == 0 (1000, 64, 36, 32 below);
# register-tile path: T % 4 != 0 (37, 50); per-column path: C > 256 or C % 8 != 0.
@pytest.mark.parametrize("B,C,T", [(32, 256, 1000), (4, 256, 64), (2, 80, 1000), (3, 64, 36),
                                   (1, 256, 32), (5, 8, 100), (2, 256, 37), (3, 80, 50),
                                   (1, 512, 64), (2, 100, 9), (1, 1024, 5)])
@pytest.mark.parametrize("act", [O.ACT_MISH, O.ACT_NONE])
def test_layernorm_channels_bct(ops, B, C, T, act):
    rng = np.random.default_rng(B * 1000 + C + T)
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    mask = (rng.random((B, T)) > 0.1).astype(np.float32)
    ref = O.layernorm_channels(x, g, b, EPS, mask, O.BCT, act)
    got = ops.layernorm_channels(dev(x), dev(g), dev(b), EPS, dev(mask), "BCT", act)
    assert_close_f32(host(got), ref, what=f"bct {B}x{C}x{T}")


@pytest.mark.parametrize("B,C,T", [(32, 256, 1000), (2, 80, 33), (1, 100, 7)])
def test_layernorm_channels_btc(ops, B, C, T):
    rng = np.random.default_rng(C + T)
    x = rng.standard_normal((B, T, C)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    ref = O.layernorm_channels(x, g, b, EPS, None, O.BTC, O.ACT_MISH)
    got = ops.layernorm_channels(dev(x), dev(g), dev(b), EPS, None, "BTC", "mish")
    assert_close_f32(host(got), ref, what="btc")


def test_layernorm_channels_silu_gelu_acts(ops):
    rng = np.random.default_rng(21)
    x = rng.standard_normal((3, 128, 96)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    for act, name in ((O.ACT_SILU, "silu"), (O.ACT_GELU, "gelu")):
        ref = O.layernorm_channels(x, g, None, EPS, None, O.BCT, act)
        assert_close_f32(host(ops.layernorm_channels(dev(x), dev(g), None, EPS, None, "BCT",
                                                     name)), ref, what=name)


# Causal block tail (conv bias + transpose + LN over C + act + mask): TMA
# kernel for T % 4 == 0, T >= 16, C in {32, 64, 128, 256}; one thread per
# column otherwise (T 45, 12; C 80, 100, 512).
@pytest.mark.parametrize("B,C,T", [(32, 256, 1000), (4, 256, 64), (3, 128, 36), (2, 64, 100),
                                   (1, 32, 16), (2, 256, 45), (3, 80, 40), (1, 100, 12),
                                   (1, 512, 20), (5, 256, 1012)])
@pytest.mark.parametrize("act,with_bias,with_mask", [(O.ACT_MISH, True, True),
                                                     (O.ACT_NONE, False, False),
                                                     (O.ACT_MISH, True, False)])
def test_causal_block1d_tail(ops, B, C, T, act, with_bias, with_mask):
    rng = np.random.default_rng(B * 7 + C + T)
    x = (1.5 * rng.standard_normal((B, C, T)) + 0.2).astype(np.float32)
    cb = (0.5 * rng.standard_normal(C)).astype(np.float32) if with_bias else None
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C)).astype(np.float32)
    mask = (rng.random((B, T)) > 0.1).astype(np.float32) if with_mask else None
    ref = O.causal_block1d_tail(x, cb, g, b, EPS, mask, act)
    got = ops.causal_block1d_tail(dev(x), None if cb is None else dev(cb), dev(g), dev(b), EPS,
                                  None if mask is None else dev(mask), act)
    assert got.shape == (B, T, C)
    assert_close_f32(host(got), ref, what=f"causal tail {B}x{C}x{T}")


def test_causal_block1d_tail_misaligned_and_equivalent_to_the_node_chain(ops):
    """A misaligned x takes the per-column kernel; both kernels equal the
    unfused chain (bias add, transpose copy, LN over C in [B][T][C])."""
    rng = np.random.default_rng(9)
    B, C, T = 3, 256, 200
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    cb = rng.standard_normal(C).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    mask = (rng.random((B, T)) > 0.2).astype(np.float32)
    fused = host(ops.causal_block1d_tail(dev(x), dev(cb), dev(g), None, EPS, dev(mask)))
    buf = torch.zeros(x.size + 1, device="cuda")
    buf[1:] = dev(x.reshape(-1))
    mis = host(ops.causal_block1d_tail(buf[1:].view(B, C, T), dev(cb), dev(g), None, EPS,
                                       dev(mask)))
    h = ops.bias_act(dev(x).view(B * C, T), dev(cb), None, axis="ne1")      # + conv_bias[c]
    h_btc = h.view(B, C, T).transpose(1, 2).contiguous()
    chain = host(ops.layernorm_channels(h_btc, dev(g), None, EPS, dev(mask), "BTC", "mish"))
    ref = O.causal_block1d_tail(x, cb, g, None, EPS, mask)
    for y, what in ((fused, "fused"), (mis, "misaligned"), (chain, "node chain")):
        assert_close_f32(y, ref, what=what)


def test_device_error_word_clear_after_normal_runs(ops):
    import ctypes
    from chatterbox_amdvulkan_b200 import _lib
    x = torch.randn((2, 256, 64), device="cuda")
    ops.layernorm_channels(x, None, None)
    ops.causal_block1d_tail(x, None, None, None)   # TMA load + swizzled TMA store kernel
    flags = ctypes.c_int32(-1)
    _lib.call("cbx_device_errors", ctypes.byref(flags),
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert flags.value == 0


def test_layernorm_channels_in_place(ops):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((4, 256, 100)).astype(np.float32)
    g = np.ones(256, np.float32)
    ref = O.layernorm_channels(x, g, None, EPS, None, O.BCT, O.ACT_MISH)
    xt = dev(x)
    ops.layernorm_channels(xt, dev(g), None, EPS, None, "BCT", "mish", out=xt)
    assert_close_f32(host(xt), ref)


# --------------------------------------------------------------- timestep --

@pytest.mark.parametrize("act", [O.ACT_NONE, O.ACT_SILU])
@pytest.mark.parametrize("dim", [320, 9, 64])
def test_timestep_embed(ops, act, dim):
    rng = np.random.default_rng(3)
    t = np.concatenate([[0.0, 1.0], rng.random(30)]).astype(np.float32)
    ref = O.timestep_embed(t, dim, 1000.0, act)
    got = ops.sinusoidal_pos_emb(dev(t), dim, 1000.0, act={0: None, 2: "silu"}[act],
                                 freqs=dev(O.sinusoid_freqs(dim)))
    assert_close_f32(host(got), ref, what="timestep")


def test_sinusoid_freqs_host_table_matches_oracle(ops):
    for dim in (4, 9, 320, 1024):
        assert np.array_equal(ops.sinusoid_freqs(dim), O.sinusoid_freqs(dim))


# ------------------------------------------------------------------ snake --

@pytest.mark.parametrize("C,T", [(256, 4000), (128, 20000), (64, 60000), (64, 101), (5, 7),
                                 (3, 6)])
def test_snake_bct(ops, C, T):
    rng = np.random.default_rng(C + T)
    B = 2
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    alpha = np.exp(0.3 * rng.standard_normal(C)).astype(np.float32)
    inv = O.snake_alpha_inv(alpha)
    ref = O.snake(x, alpha, inv)
    got = ops.snake(dev(x), dev(alpha), dev(inv))
    assert_close_f32(host(got), ref, what="snake")
    got2 = ops.snake(dev(x), dev(alpha), None)   # alpha_inv formed on the device
    assert np.array_equal(host(got2), host(got))


@pytest.mark.parametrize("C,T", [(64, 300), (6, 10)])
def test_snake_btc(ops, C, T):
    rng = np.random.default_rng(C)
    x = rng.standard_normal((2, T, C)).astype(np.float32) * 3
    alpha = np.exp(0.3 * rng.standard_normal(C)).astype(np.float32)
    ref = O.snake(x, alpha, None, layout=O.BTC)
    assert_close_f32(host(ops.snake(dev(x), dev(alpha), None, layout="BTC")), ref)


def test_snake_config4_full_size_sampled(ops):
    """Config 4 stage 2 at full size (B=16, C=64, T=60000); 64 rows checked."""
    rng = np.random.default_rng(4)
    B, C, T = 16, 64, 60000
    xt = torch.randn((B, C, T), device="cuda")
    alpha = np.exp(0.3 * rng.standard_normal(C)).astype(np.float32)
    inv = O.snake_alpha_inv(alpha)
    y = ops.snake(xt, dev(alpha), dev(inv))
    for bi, c in zip(rng.integers(0, B, 64), rng.integers(0, C, 64)):
        xr = host(xt[bi, c]).reshape(1, 1, T)
        ref = O.snake(xr, alpha[c:c + 1], inv[c:c + 1])
        assert_close_f32(host(y[bi, c]).reshape(1, 1, T), ref, what="snake cfg4")


# ------------------------------------------------------------- embedding --

@pytest.mark.parametrize("tab_t,out_t", [(O.F32, O.F32), (O.F16, O.F32), (O.BF16, O.BF16),
                                         (O.BF16, O.F32), (O.F32, O.BF16), (O.F16, O.F16)])
def test_embed_gather_add_bit_exact(ops, tab_t, out_t):
    rng = np.random.default_rng(0)
    V, P, H, n = 6563, 4096, 1024, 512
    tok = O.to_type((0.02 * rng.standard_normal((V, H))).astype(np.float32), tab_t)
    pos = O.to_type((0.02 * rng.standard_normal((P, H))).astype(np.float32), tab_t)
    ids = rng.integers(0, 6561, n).astype(np.int32)
    ids[:2] = [0, V - 1]
    ref, err = O.embed_gather_add(tok, tab_t, ids, pos, tab_t, pos_offset=0, out_t=out_t)
    assert err == 0
    got = ops.embed_gather_add(dev(tok, tab_t), torch.from_numpy(ids).cuda(), dev(pos, tab_t),
                               n_past=0, out_dtype={O.F32: torch.float32,
                                                    O.BF16: torch.bfloat16,
                                                    O.F16: torch.float16}[out_t])
    assert np.array_equal(host(got), ref)


def test_embed_config2_full_size(ops):
    """Config 2: 65536 rows (64 x 1024 positions), bf16 tables and output."""
    rng = np.random.default_rng(2)
    V, P, H = 6563, 4096, 1024
    tok = O.to_type((0.02 * rng.standard_normal((V, H))).astype(np.float32), O.BF16)
    pos = O.to_type((0.02 * rng.standard_normal((P, H))).astype(np.float32), O.BF16)
    ids = rng.integers(0, 6561, 65536).astype(np.int32)
    pid = (np.arange(65536) % 1024).astype(np.int32)
    ref, _ = O.embed_gather_add(tok, O.BF16, ids, pos, O.BF16, pos_ids=pid, out_t=O.BF16)
    got = ops.embed_gather_add(dev(tok, O.BF16), torch.from_numpy(ids).cuda(),
                               dev(pos, O.BF16), pos_ids=torch.from_numpy(pid).cuda(),
                               out_dtype=torch.bfloat16)
    assert np.array_equal(host(got), ref)


@pytest.mark.parametrize("t", [O.BF16, O.F16])
def test_embed_packed_16bit_add_equals_f32_sum_on_all_bit_patterns(ops, t):
    """Same 16-bit type in and out takes the packed bf16x2 / f16x2 add: on
    random bit patterns (every exponent, subnormals, +-0, +-inf, NaN) it
    returns the bits of the f32 sum rounded once, NaN where the sum is NaN."""
    rng = np.random.default_rng(21 + t)
    V, P, H, n = 300, 200, 1024, 700
    tok = rng.integers(0, 1 << 16, (V, H), dtype=np.uint16)
    pos = rng.integers(0, 1 << 16, (P, H), dtype=np.uint16)
    # planted pairs: exact ties at the rounding point, opposite zeros, cancellation
    tok[:4, :3] = 0x8000
    pos[:4, :3] = 0x0000
    ids = rng.integers(0, V, n).astype(np.int32)
    ids[:4] = [0, 1, 2, 3]
    pid = rng.integers(0, P, n).astype(np.int32)
    pid[:4] = [0, 1, 2, 3]
    ref, _ = O.embed_gather_add(tok, t, ids, pos, t, pos_ids=pid, out_t=t)
    tdt = torch.bfloat16 if t == O.BF16 else torch.float16
    got = host(ops.embed_gather_add(dev(tok, t), torch.from_numpy(ids).cuda(), dev(pos, t),
                                    pos_ids=torch.from_numpy(pid).cuda(), out_dtype=tdt))
    ref_f = O.to_f32(ref, t)
    nan = np.isnan(ref_f)
    assert np.array_equal(np.isnan(O.to_f32(got, t)), nan)
    assert np.array_equal(got[~nan], ref[~nan])
    # without a position table the rows are copied bit for bit
    got2 = host(ops.embed_gather_add(dev(tok, t), torch.from_numpy(ids).cuda(), out_dtype=tdt))
    assert np.array_equal(got2, tok[ids])


@pytest.mark.parametrize("t", [O.BF16, O.F16])
@pytest.mark.parametrize("H,n,form", [(1024, 5003, "pos_ids"), (520, 2400, "n_past"),
                                      (8, 3000, "no_pos"), (8192, 2371, "pos_ids"),
                                      (64, 148 * 1024 + 77, "n_past")])
def test_embed_many_rows_16bit(ops, t, H, n, form):
    """Same 16-bit type in and out with enough rows to fill the GPU (several
    rows per warp, partial last blocks): rows of 16 B to 16 KB, position ids,
    an n_past offset whose last rows run past the table, no position table,
    planted out-of-range ids and positions (zero rows, flags): bit-exact
    against the oracle."""
    rng = np.random.default_rng(H + n + t)
    V, P = 300, max(4096, n + 64)
    tok = O.to_type((0.02 * rng.standard_normal((V, H))).astype(np.float32), t)
    pos = O.to_type((0.02 * rng.standard_normal((P, H))).astype(np.float32), t)
    ids = rng.integers(0, V, n).astype(np.int32)
    ids[[5, n - 1]] = [V, -3]
    pid = rng.integers(0, P, n).astype(np.int32)
    pid[[9, n // 2]] = [P, -1]
    n_past = 0
    kw = {}
    if form == "pos_ids":
        kw["pos_ids"] = torch.from_numpy(pid).cuda()
        ref, err_ref = O.embed_gather_add(tok, t, ids, pos, t, pos_ids=pid, out_t=t)
    elif form == "n_past":
        n_past = P - n + 40 if n < P else 0   # the last rows run past the table
        kw["n_past"] = n_past
        ref, err_ref = O.embed_gather_add(tok, t, ids, pos, t, pos_offset=n_past, out_t=t)
    else:
        ref, err_ref = O.embed_gather_add(tok, t, ids, None, out_t=t)
    tdt = torch.bfloat16 if t == O.BF16 else torch.float16
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = ops.embed_gather_add(dev(tok, t), torch.from_numpy(ids).cuda(),
                               None if form == "no_pos" else dev(pos, t), out_dtype=tdt,
                               err_word=err, **kw)
    assert np.array_equal(host(got), ref)
    assert int(err.item()) == err_ref and err_ref & 1


def test_embed_mixed_types_and_no_pos(ops):
    rng = np.random.default_rng(9)
    tok = O.to_type((0.02 * rng.standard_normal((50, 72))).astype(np.float32), O.F16)
    pos = (0.02 * rng.standard_normal((40, 72))).astype(np.float32)
    ids = rng.integers(0, 50, 30).astype(np.int32)
    ref, _ = O.embed_gather_add(tok, O.F16, ids, pos, O.F32, pos_offset=3, out_t=O.F32)
    got = ops.embed_gather_add(dev(tok, O.F16), torch.from_numpy(ids).cuda(), dev(pos),
                               n_past=3)
    assert np.array_equal(host(got), ref)
    ref2, _ = O.embed_gather_add(tok, O.F16, ids, None, out_t=O.F32)
    got2 = ops.embed_gather_add(dev(tok, O.F16), torch.from_numpy(ids).cuda())
    assert np.array_equal(host(got2), ref2)


def test_embed_out_of_range_ids_flagged_not_read(ops):
    rng = np.random.default_rng(10)
    tok = (0.02 * rng.standard_normal((100, 256))).astype(np.float32)
    pos = (0.02 * rng.standard_normal((64, 256))).astype(np.float32)
    ids = rng.integers(0, 100, 40).astype(np.int32)
    ids[3], ids[7] = 100, -5
    ref, err_ref = O.embed_gather_add(tok, O.F32, ids, pos, O.F32, pos_offset=30)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = ops.embed_gather_add(dev(tok), torch.from_numpy(ids).cuda(), dev(pos), n_past=30,
                               err_word=err)
    assert np.array_equal(host(got), ref)
    assert int(err.item()) == err_ref == 3


# -------------------------------------------------------------- C ABI misc --

def test_errors_do_not_launch(ops):
    import ctypes
    from chatterbox_amdvulkan_b200 import CbxError, _lib
    x = torch.zeros(16, device="cuda")
    with pytest.raises(CbxError, match="INVALID_ARG"):
        ops.layernorm_channels(x.view(1, 4, 4), None, None, layout=5)
    with pytest.raises(CbxError, match="UNSUPPORTED_DTYPE"):
        _lib.call("cbx_gelu_tanh", ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                  16, 99, None)
    torch.cuda.synchronize()
    assert torch.all(x == 0)


def test_zero_sizes_are_noops(ops):
    x = torch.zeros(0, device="cuda")
    assert ops.gelu(x).numel() == 0
    assert ops.add_layernorm(torch.zeros((0, 1024), device="cuda"), None, None, None).numel() == 0


# ------------------------------------------------------ epilogue neighbours --

def test_epilogue_neighbours_match_reference_goldens(ops, golden):
    g = golden
    x = dev(g["gerf_x"])
    assert_close_f32(host(ops.gelu_erf(x)), g["gerf_y"], what="gelu_erf")
    assert_close_f32(host(ops.bias_act(x, None, "elu")), g["elu_y"], what="elu")
    assert_close_f32(host(ops.bias_act(x, None, "leaky_relu", act_param=0.1)), g["lrelu01_y"],
                     what="leaky 0.1")
    assert_close_f32(host(ops.bias_act(x, None, "leaky_relu", act_param=0.01)),
                     g["lrelu001_y"], what="leaky 0.01")
    assert_close_f32(host(ops.bias_act(dev(g["fc_h"]), dev(g["fc_b"]), "gelu")), g["fc_y"],
                     what="fc bias + gelu")
    assert np.array_equal(host(ops.bias_act(dev(g["cb_x"]), dev(g["cb_b"]), None, axis="ne1")),
                          g["cb_y"])
    y = ops.sum3_scale(dev(g["rb_r0"]), dev(g["rb_r1"]), dev(g["rb_r2"]), np.float32(1 / 3))
    assert_close_f32(host(y), g["rb_y"], what="resblock mean")


@pytest.mark.parametrize("t", [O.F32, O.BF16, O.F16])
def test_gelu_erf_parity(ops, t):
    rng = np.random.default_rng(13)
    x32 = normal_with_outliers(rng, (5003,), frac=0.02) * 3.0
    x32[:8] = [0.0, -0.0, 20.0, -20.0, -6.0, 6.0, np.inf, -np.inf]
    xq = O.to_type(x32, t)
    ref = O.gelu_erf(O.to_f32(xq, t))
    _check_typed(ops.gelu_erf(dev(xq, t)), ref, t, f"gelu_erf {t}")


@pytest.mark.parametrize("name,t", [("gelu", O.BF16), ("silu", O.F16), ("mish", O.BF16),
                                    ("gelu_erf", O.F32)])
def test_activation_few_iterations_per_thread(ops, name, t):
    """Launches of a few grid-stride iterations per thread at 4 CTAs per SM
    (the shape of a multi-GPU shard of configs[2]'s GELU), ragged tail
    included: same results as the oracle."""
    rng = np.random.default_rng(17)
    n = 4096 * 2048 + 13
    x32 = (rng.standard_normal(n) * 3.0).astype(np.float32)
    xq = O.to_type(x32, t)
    fn = {"gelu": O.gelu_tanh, "silu": O.silu, "mish": O.mish, "gelu_erf": O.gelu_erf}[name]
    ref = fn(O.to_f32(xq, t))
    _check_typed(getattr(ops, name)(dev(xq, t)), ref, t, f"{name} {t} n={n}")


_ACTS = [("none", O.ACT_NONE, 0.0), ("gelu", O.ACT_GELU, 0.0), ("gelu_erf", O.ACT_GELU_ERF, 0.0),
         ("silu", O.ACT_SILU, 0.0), ("mish", O.ACT_MISH, 0.0), ("elu", O.ACT_ELU, 0.0),
         ("leaky_relu", O.ACT_LEAKY_RELU, 0.1)]


@pytest.mark.parametrize("name,act,param", _ACTS)
@pytest.mark.parametrize("axis", ["ne0", "ne1", None])
@pytest.mark.parametrize("t", [O.F32, O.BF16])
def test_bias_act_parity(ops, name, act, param, axis, t):
    rng = np.random.default_rng(act * 7 + (axis == "ne1"))
    rows, H = 96, 512
    x = O.to_type(normal_with_outliers(rng, (rows, H)) * 2.0, t)
    if axis == "ne0":
        bias = rng.standard_normal(H).astype(np.float32)
    elif axis == "ne1":
        bias = rng.standard_normal(32).astype(np.float32)     # rows = 3 items x 32 channels
    else:
        bias = None
    ref = O.bias_act(O.to_f32(x, t), bias, O.BIAS_NE1 if axis == "ne1" else O.BIAS_NE0, act,
                     param)
    got = ops.bias_act(dev(x, t), None if bias is None else dev(bias), name,
                       axis=axis or "ne0", act_param=param)
    _check_typed(got, ref, t, f"bias_act {name} {axis} {t}")


def test_bias_act_ragged_misaligned_and_large(ops):
    rng = np.random.default_rng(14)
    # ragged hidden (not a multiple of the vector width): the scalar path
    x = rng.standard_normal((7, 333)).astype(np.float32)
    b = rng.standard_normal(333).astype(np.float32)
    assert_close_f32(host(ops.bias_act(dev(x), dev(b), "gelu")),
                     O.bias_act(x, b, O.BIAS_NE0, O.ACT_GELU), what="ragged")
    # misaligned view (4-byte offset)
    buf = dev(np.concatenate([[0.0], x.reshape(-1)]).astype(np.float32))
    got = ops.bias_act(buf[1:].view(7, 333), dev(b), "gelu")
    assert_close_f32(host(got), O.bias_act(x, b, O.BIAS_NE0, O.ACT_GELU), what="misaligned")
    # T3 fc epilogue shape at full width (rows sampled), bf16 in/out
    rows, H = 4096, 4096
    xt = torch.randn((rows, H), device="cuda").to(torch.bfloat16)
    bt = 0.5 * torch.randn(H, device="cuda")
    y = ops.bias_act(xt, bt, "gelu")
    pick = np.sort(rng.choice(rows, 256, replace=False))
    ref = O.bias_act(O.to_f32(host(xt[pick]), O.BF16), host(bt), O.BIAS_NE0, O.ACT_GELU)
    assert_within_bf16_ulps(host_f32(y[pick]), ref, what="fc epilogue bf16")


@pytest.mark.parametrize("t", [O.F32, O.BF16, O.F16])
@pytest.mark.parametrize("n", [64 * 101, 16 * 256 * 4000 // 8, 1001])
def test_sum3_scale_bit_exact(ops, t, n):
    rng = np.random.default_rng(n)
    a, b, c = (O.to_type(rng.standard_normal(n).astype(np.float32), t) for _ in range(3))
    s = np.float32(1.0 / 3.0)
    ref = O.sum3_scale(a, b, c, s, t)
    got = ops.sum3_scale(dev(a, t), dev(b, t), dev(c, t), float(s))
    assert np.array_equal(host(got), ref)


def test_sum3_scale_misaligned(ops):
    rng = np.random.default_rng(15)
    a, b, c = (rng.standard_normal(1000).astype(np.float32) for _ in range(3))
    bufs = [dev(np.concatenate([[0.0], v]).astype(np.float32))[1:] for v in (a, b, c)]
    got = ops.sum3_scale(*bufs, scale=0.25)
    assert np.array_equal(host(got), O.sum3_scale(a, b, c, 0.25))
