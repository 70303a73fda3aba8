"""Pin the CPU oracle (oracle/cbx_oracle.c) against the reference's own NumPy
oracles (fixtures written by tests/golden/make_golden.py from
scripts/reference_t3_forward.py, reference_cfm_decoder.py and
reference_hift_vocoder.py), and check its host logic.  CPU only."""
import math

import numpy as np
import pytest

import oracle as O
from conftest import assert_close_f32, assert_within_bf16_ulps


def test_gelu_tanh_matches_reference(golden):
    assert_close_f32(O.gelu_tanh(golden["gelu_x"]), golden["gelu_y"], what="gelu")


def test_add_layernorm_matches_reference(golden):
    s, y = O.add_layernorm(golden["ln_x"], golden["ln_r"], golden["ln_w"], golden["ln_b"], 1e-5)
    assert np.array_equal(s, golden["ln_s"])  # the residual sum is one IEEE add
    assert_close_f32(y, golden["ln_y"], what="ln")


def test_layernorm_ragged_hidden_matches_reference(golden):
    _, y = O.add_layernorm(golden["ln2_x"], None, golden["ln2_w"], golden["ln2_b"], 1e-5)
    assert_close_f32(y, golden["ln2_y"], what="ln ragged")


def test_silu_mish_match_reference(golden):
    assert_close_f32(O.silu(golden["act_x"]), golden["silu_y"], what="silu")
    assert_close_f32(O.mish(golden["act_x"]), golden["mish_y"], what="mish")


def test_cfm_block_tail_matches_reference(golden):
    y = O.layernorm_channels(golden["cfm_x"], golden["cfm_w"], golden["cfm_b"], 1e-5,
                             golden["cfm_mask"], layout=O.BCT, act=O.ACT_MISH)
    assert_close_f32(y, golden["cfm_y"], what="cfm ln+mish+mask")
    y = O.layernorm_channels(golden["cfm_x"], golden["cfm_w"], golden["cfm_b"], 1e-5, None,
                             layout=O.BCT, act=O.ACT_NONE)
    assert_close_f32(y, golden["cfm_ln_only"], what="cfm ln")


def test_causal_block1d_tail_matches_reference(golden):
    """The causal conv's epilogue + block tail (conv bias, LN over C, Mish,
    mask; reference_cfm_decoder.py:199-202, :238-251), output in the engine's
    [B][T][C]."""
    g = golden
    y = O.causal_block1d_tail(g["cbt_x"], g["cbt_cb"], g["cbt_w"], g["cbt_b"], 1e-5,
                              g["cbt_mask"])
    assert y.shape == g["cbt_y"].shape
    assert_close_f32(y, g["cbt_y"], what="causal block tail")
    # masked steps are exactly zero
    assert np.all(y[0, -9:, :] == 0.0)


def test_cfm_btc_layout_equals_bct(golden):
    x = golden["cfm_x"]
    y_bct = O.layernorm_channels(x, golden["cfm_w"], golden["cfm_b"], 1e-5, golden["cfm_mask"])
    y_btc = O.layernorm_channels(np.ascontiguousarray(x.transpose(0, 2, 1)), golden["cfm_w"],
                                 golden["cfm_b"], 1e-5, golden["cfm_mask"], layout=O.BTC)
    assert np.array_equal(y_bct, y_btc.transpose(0, 2, 1))


def _f32_ulp(a):
    a = np.abs(np.asarray(a, np.float64))
    return 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -126))) - 23)


def test_sinusoid_matches_reference(golden):
    t = golden["sin_t"]
    # scale 1: |a| <= 1, the frequency table's last-ulp differences do not show.
    assert_close_f32(O.timestep_embed(t, 320, 1.0), golden["sin_y_scale1"], what="sin scale 1")
    # scale 1000: the engine's C++ f32 frequency expression (cfm_decoder.cpp:52-56)
    # and NumPy's (reference_cfm_decoder.py:220-222) differ by <= 1 ulp in some
    # entries; at |a| up to 1000 that moves sin/cos by up to 2 ulp(a).
    fr = O.sinusoid_freqs(320)
    a = (np.float32(1000.0) * t)[:, None].astype(np.float32) * np.concatenate([fr, fr])[None, :]
    got = O.timestep_embed(t, 320, 1000.0)
    ref = golden["sin_y"]
    bound = 1e-6 + 1e-5 * np.abs(ref) + 2.0 * _f32_ulp(a)
    assert np.all(np.abs(got - ref) <= bound)
    silu = O.timestep_embed(t, 320, 1000.0, act=O.ACT_SILU)
    assert np.all(np.abs(silu - golden["sin_silu_y"]) <= bound)


def test_sinusoid_freqs_follow_engine_expression():
    fr = O.sinusoid_freqs(320)
    half = 160
    factor = np.float32(math.log(10000.0)) / np.float32(half - 1)  # f32 as the engine
    assert fr[0] == 1.0
    # NumPy's reference expression agrees to 1 ulp.
    npfr = np.exp(np.arange(half, dtype=np.float32) * -(math.log(10000.0) / (half - 1)))
    assert np.max(np.abs(fr.view(np.int32) - npfr.view(np.int32))) <= 1
    assert np.all(np.diff(fr) < 0) and factor > 0
    with pytest.raises(ValueError):
        O.sinusoid_freqs(2)


def test_sinusoid_odd_dim_zero_tail():
    y = O.timestep_embed(np.array([0.25], np.float32), 9, 1000.0)
    assert y.shape == (1, 9) and y[0, 8] == 0.0


def test_snake_matches_reference(golden):
    y = O.snake(golden["snake_x"], golden["snake_alpha"])
    assert_close_f32(y, golden["snake_y"], what="snake")
    inv = O.snake_alpha_inv(golden["snake_alpha"])
    assert np.array_equal(O.snake(golden["snake_x"], golden["snake_alpha"], inv), y)


def test_snake_btc_equals_bct(golden):
    x = golden["snake_x"]
    y = O.snake(x, golden["snake_alpha"])
    y2 = O.snake(np.ascontiguousarray(x.transpose(0, 2, 1)), golden["snake_alpha"], layout=O.BTC)
    assert np.array_equal(y, y2.transpose(0, 2, 1))


def test_embed_gather_add_bit_exact(golden):
    n_past = int(golden["emb_npast"][0])
    out, err = O.embed_gather_add(golden["emb_tok"], O.F32, golden["emb_ids"], golden["emb_pos"],
                                  O.F32, pos_offset=n_past)
    assert err == 0 and np.array_equal(out, golden["emb_y"])
    out, err = O.embed_gather_add(golden["emb_tok16"], O.F16, golden["emb_ids"],
                                  golden["emb_pos16"], O.F16, pos_offset=n_past)
    assert err == 0 and np.array_equal(out, golden["emb16_y"])
    # explicit position ids == offset form
    pid = np.arange(n_past, n_past + golden["emb_ids"].size, dtype=np.int32)
    out2, _ = O.embed_gather_add(golden["emb_tok16"], O.F16, golden["emb_ids"],
                                 golden["emb_pos16"], O.F16, pos_ids=pid)
    assert np.array_equal(out2, out)


def test_embed_out_of_range_rows_are_zero_and_flagged(golden):
    ids = golden["emb_ids"].copy()
    ids[2] = 97          # == n_tok_rows
    ids[5] = -1
    out, err = O.embed_gather_add(golden["emb_tok"], O.F32, ids, golden["emb_pos"], O.F32,
                                  pos_offset=40)       # rows 10.. run past 50 positions
    assert err == (1 | 2)
    assert not out[2].any() and not out[5].any() and not out[15].any()
    assert np.array_equal(out[0], golden["emb_tok"][ids[0]] + golden["emb_pos"][40])


@pytest.mark.parametrize("t", [O.BF16, O.F16])
def test_dtype_conversions_match_numpy(t):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 100,
                        np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 1e-8, 3e38],
                                 np.float32)])
    q = O.to_type(x, t)
    back = O.to_f32(q, t)
    if t == O.F16:
        ref = x.astype(np.float16).astype(np.float32)
        assert np.array_equal(back, ref)
    else:
        # bf16 = top 16 bits after round-to-nearest-even
        u = x.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        assert np.array_equal(q, r)
    assert np.isnan(O.to_f32(O.to_type(np.array([np.nan], np.float32), t), t)[0])


def test_bf16_layernorm_within_two_ulp_of_f32(golden):
    x = golden["ln_x"]
    r = golden["ln_r"]
    xb, rb = O.to_type(x, O.BF16), O.to_type(r, O.BF16)
    s, y = O.add_layernorm(xb, rb, golden["ln_w"], golden["ln_b"], 1e-5, in_t=O.BF16,
                           out_t=O.BF16)
    s32 = O.to_f32(xb, O.BF16) + O.to_f32(rb, O.BF16)
    assert np.array_equal(s, O.to_type(s32, O.BF16))
    _, y_ref = O.add_layernorm(s32, None, golden["ln_w"], golden["ln_b"], 1e-5)
    assert_within_bf16_ulps(O.to_f32(y, O.BF16), y_ref, ulps=1, what="bf16 ln")


def test_bad_arguments_rejected():
    with pytest.raises(ValueError):
        O.snake(np.zeros((1, 4, 4), np.float32), np.ones(4, np.float32), layout=7)
    with pytest.raises(ValueError):
        O.timestep_embed(np.zeros(2, np.float32), 320, act=O.ACT_MISH)


def test_epilogue_neighbours_match_reference(golden):
    g = golden
    assert_close_f32(O.gelu_erf(g["gerf_x"]), g["gerf_y"], what="gelu_erf")
    assert_close_f32(O.bias_act(g["gerf_x"], act=O.ACT_ELU), g["elu_y"], what="elu")
    assert_close_f32(O.bias_act(g["gerf_x"], act=O.ACT_LEAKY_RELU, param=0.1), g["lrelu01_y"],
                     what="leaky 0.1")
    assert_close_f32(O.bias_act(g["gerf_x"], act=O.ACT_LEAKY_RELU, param=0.01),
                     g["lrelu001_y"], what="leaky 0.01")
    # fc bias then GELU-tanh: the sum is one IEEE add, then the activation
    assert_close_f32(O.bias_act(g["fc_h"], g["fc_b"], O.BIAS_NE0, O.ACT_GELU), g["fc_y"],
                     what="fc bias + gelu")
    # conv bias per channel row of a (C, T) block
    assert np.array_equal(O.bias_act(g["cb_x"], g["cb_b"], O.BIAS_NE1), g["cb_y"])
    # ResBlock average: the engine multiplies by 1/3f, NumPy divides by 3 (<= 1 ulp apart)
    assert_close_f32(O.sum3_scale(g["rb_r0"], g["rb_r1"], g["rb_r2"], np.float32(1.0 / 3.0)),
                     g["rb_y"], what="resblock mean")


# ------------------------------------------------ HiFT source and STFT/iSTFT --

def test_hann_window_matches_reference(golden):
    # engine f32 host expression (cosf) vs NumPy's f32 cos: <= 1 ulp apart
    assert np.max(np.abs(O.hann_window(16) - golden["hann16"])) <= 6e-8
    assert O.hann_window(16)[0] == 0.0


def test_nsf_source_matches_reference(golden):
    g = golden
    y = O.nsf_source(g["nsf_f0"][None], 480, g["nsf_phase"], g["nsf_noise"], g["nsf_lw"],
                     float(g["nsf_lb"][0]))
    assert_close_f32(y, g["nsf_y"], what="nsf source")


def test_nsf_phase_of_the_fundamental_is_zero(golden):
    g = golden
    ph = g["nsf_phase"].copy()
    ph[0, 0] = 1.234          # ignored: the engine forces phase_vec[0] = 0
    y = O.nsf_source(g["nsf_f0"][None], 480, ph, g["nsf_noise"], g["nsf_lw"],
                     float(g["nsf_lb"][0]))
    assert np.array_equal(y, O.nsf_source(g["nsf_f0"][None], 480, g["nsf_phase"], g["nsf_noise"],
                                          g["nsf_lw"], float(g["nsf_lb"][0])))


def test_stft_matches_reference(golden):
    g = golden
    y = O.stft(g["stft_x"], 16, 4, g["hann16"], layout=O.BCT)
    # NumPy's rfft runs in f32 here, the engine's DFT in double
    assert np.max(np.abs(y - g["stft_y"])) <= 1e-6
    yb = O.stft(g["stft_x"], 16, 4, g["hann16"], layout=O.BTC)
    assert np.array_equal(yb, y.transpose(0, 2, 1))


def test_istft_post_matches_reference(golden):
    g = golden
    y = O.istft_post(g["istft_post"][None], 16, 4, g["hann16"], layout=O.BCT)
    assert_close_f32(y, g["istft_y"], what="istft")
    yb = O.istft_post(np.ascontiguousarray(g["istft_post"].T)[None], 16, 4, g["hann16"],
                      layout=O.BTC)
    assert np.array_equal(yb, y)


def test_stft_scaling_and_linearity():
    rng = np.random.default_rng(3)
    x = (0.4 * rng.standard_normal((1, 400))).astype(np.float32)
    z = (0.4 * rng.standard_normal((1, 400))).astype(np.float32)
    sx = O.stft(x)
    # scaling by a power of two is exact through every f32 and f64 operation
    assert np.array_equal(O.stft(2.0 * x), 2.0 * sx)
    assert np.max(np.abs(O.stft(x + z) - (sx + O.stft(z)))) <= 2e-6


def test_hift_dsp_bad_arguments():
    with pytest.raises(ValueError):
        O.stft(np.zeros((1, 8), np.float32), 16, 4)       # T <= n_fft / 2
    with pytest.raises(ValueError):
        O.istft_post(np.zeros((1, 4, 18), np.float32), 15, 4)


# ------------------------------------------------------ T3 QKV epilogue --

def test_qkv_kv_append_matches_reference_split(golden):
    g = golden
    D = g["kv_q"].shape[1]
    ck = np.zeros((16, D), np.float32)
    cv = np.zeros((16, D), np.float32)
    q, err = O.qkv_kv_append(g["kv_h"], g["kv_b"], ck, cv, O.F32, pos_offset=3, max_context=16)
    assert err == 0
    assert np.array_equal(q, g["kv_q"])
    assert np.array_equal(ck[3:8], g["kv_k"]) and np.array_equal(cv[3:8], g["kv_v"])
    assert not ck[:3].any() and not ck[8:].any()


def test_qkv_kv_append_per_stream_positions_and_oob():
    rng = np.random.default_rng(4)
    n, D, ctx = 4, 8, 6
    x = rng.standard_normal((n, 3 * D)).astype(np.float32)
    ck = np.full((n, ctx, D), 7.0, np.float32)
    cv = np.full((n, ctx, D), 7.0, np.float32)
    pos = np.array([0, 5, 6, -1], np.int32)     # the last two are out of range
    q, err = O.qkv_kv_append(x, None, ck, cv, O.F32, positions=pos, slab_stride=ctx * D,
                             max_context=ctx)
    assert err == 2 and np.array_equal(q, x[:, :D])
    assert np.array_equal(ck[0, 0], x[0, D:2 * D]) and np.array_equal(cv[1, 5], x[1, 2 * D:])
    assert np.all(ck[2:] == 7.0) and np.all(cv[2:] == 7.0)
    # f16 cache: the engine-equivalent rounding of the f32 sum
    ck16 = np.zeros((n, ctx, D), np.uint16)
    cv16 = np.zeros((n, ctx, D), np.uint16)
    O.qkv_kv_append(x, None, ck16, cv16, O.F16, positions=pos, slab_stride=ctx * D,
                    max_context=ctx)
    assert np.array_equal(ck16[0, 0], x[0, D:2 * D].astype(np.float16).view(np.uint16))


def test_t3_prefill_sequence_matches_reference(golden):
    """[cond ; speech[prompt] ; text[ids]] + wpe[:L], caught from the reference's
    own t3_forward (reference_t3_forward.py:150-172), f16 tables."""
    g = golden
    out, err = O.t3_embed_sequence(g["seq_text16"], O.F16, g["seq_text_ids"], g["seq_pos16"],
                                   O.F16, 0, g["seq_cond"], g["seq_speech16"], O.F16,
                                   g["seq_prompt_ids"])
    assert err == 0 and np.array_equal(out, g["seq_y"])
    # the same rows as the three gathers of the engine's graph, one call each
    n_p = g["seq_prompt_ids"].size
    mid, _ = O.embed_gather_add(g["seq_speech16"], O.F16, g["seq_prompt_ids"], g["seq_pos16"],
                                O.F16, pos_offset=1)
    assert np.array_equal(out[1:1 + n_p], mid)
