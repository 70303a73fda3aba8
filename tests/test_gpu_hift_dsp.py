"""GPU parity of the HiFT DSP entry points (cbx_nsf_source, cbx_stft,
cbx_istft_post) against the CPU oracle and the reference's NumPy fixtures.

Bar: f32 outputs within |gpu - ref| <= 1e-6 + 1e-5 |ref| of the oracle, which
restates the engine's host loops (hift_vocoder.cpp:465-541, :787-829,
:853-965) with its double sums."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from _gpu import dev, host
from conftest import assert_close_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


def f0_contour(rng, B, n_mel, unvoiced_frac=0.2):
    """Speech-like f0: a smooth 80-400 Hz contour per utterance with unvoiced
    (0 Hz) stretches and leading / trailing silence."""
    t = np.arange(n_mel)
    f0 = np.empty((B, n_mel), np.float32)
    for b in range(B):
        base = rng.uniform(90, 260)
        f = base * (1.0 + 0.25 * np.sin(2 * np.pi * t / rng.uniform(20, 90) + rng.uniform(0, 6)))
        f += rng.normal(0, 3, n_mel)
        uv = rng.random(n_mel) < unvoiced_frac
        uv[: rng.integers(1, 6)] = True
        uv[-rng.integers(1, 6):] = True
        f0[b] = np.where(uv, 0.0, np.clip(f, 60, 420)).astype(np.float32)
    return f0


def nsf_inputs(rng, B, n_mel, up=480):
    phase = rng.uniform(-np.pi, np.pi, (B, 9)).astype(np.float32)
    noise = rng.standard_normal((B, 9, n_mel * up)).astype(np.float32)
    lw = (0.4 * rng.standard_normal(9)).astype(np.float32)
    return phase, noise, lw


def run_nsf(ops, f0, up, phase, noise, lw, lb, sr=24000):
    return host(ops.nsf_source(dev(f0), up, dev(phase), dev(noise), lw, lb, sr))


# ------------------------------------------------------------ golden pins --

def test_gpu_dsp_matches_reference_goldens(ops, golden):
    g = golden
    y = run_nsf(ops, g["nsf_f0"][None], 480, g["nsf_phase"], g["nsf_noise"], g["nsf_lw"],
                float(g["nsf_lb"][0]))
    assert_close_f32(y, g["nsf_y"], what="nsf source")
    assert np.array_equal(ops.hann_window(16), O.hann_window(16))
    s = host(ops.stft(dev(g["stft_x"]), 16, 4, dev(g["hann16"]), layout="BCT"))
    assert np.max(np.abs(s - g["stft_y"])) <= 1e-6
    w = host(ops.istft_post(dev(g["istft_post"][None]), 16, 4, dev(g["hann16"]), layout="BCT"))
    assert_close_f32(w, g["istft_y"], what="istft")


# -------------------------------------------------------------- NSF source --

@pytest.mark.parametrize("B,n_mel,up", [(3, 60, 480), (2, 37, 100), (1, 9, 600), (4, 130, 480)])
def test_nsf_source_parity(ops, B, n_mel, up):
    rng = np.random.default_rng(100 + n_mel)
    f0 = f0_contour(rng, B, n_mel)
    phase, noise, lw = nsf_inputs(rng, B, n_mel, up)
    got = run_nsf(ops, f0, up, phase, noise, lw, 0.03)
    ref = O.nsf_source(f0, up, phase, noise, lw, 0.03)
    assert_close_f32(got, ref, what=f"nsf B={B} n_mel={n_mel} up={up}")


@pytest.mark.parametrize("up,off", [(480, 1), (99, 0), (10, 0), (17, 0), (18, 0), (480, 0)])
def test_nsf_source_both_frame_start_paths(ops, up, off):
    """The frame starts come from the separate scan kernel, parked in each
    frame's own output samples (upsample even and >= 18, output 8-byte
    aligned), or from each CTA's own replay (odd or small upsample, or an
    output 4 bytes off alignment): both equal the oracle, and the first path
    leaves no trace of the parked values in the output."""
    rng = np.random.default_rng(up + off)
    B, n_mel = 3, 41
    f0 = f0_contour(rng, B, n_mel)
    phase, noise, lw = nsf_inputs(rng, B, n_mel, up)
    buf = torch.full((B * n_mel * up + off,), 123.0, device="cuda")
    out = buf[off:].view(B, n_mel * up)
    ops.nsf_source(dev(f0), up, dev(phase), dev(noise), lw, 0.02, out=out)
    ref = O.nsf_source(f0, up, phase, noise, lw, 0.02)
    assert_close_f32(host(out), ref, what=f"nsf up={up} off={off}")


def test_nsf_source_scan_beyond_the_shared_increment_table(ops):
    """n_mel above the scan kernel's shared-memory increment table (3072
    frames): the scan forms the increments from f0 in global memory."""
    rng = np.random.default_rng(12)
    n_mel, up = 3100, 20
    f0 = f0_contour(rng, 2, n_mel, unvoiced_frac=0.1)
    phase, noise, lw = nsf_inputs(rng, 2, n_mel, up)
    got = run_nsf(ops, f0, up, phase, noise, lw, 0.01)
    ref = O.nsf_source(f0, up, phase, noise, lw, 0.01)
    assert_close_f32(got, ref, what="nsf n_mel 3100")


def test_nsf_source_long_utterance_exact_phase(ops):
    """40 s at 24 kHz: the engine's sequential double phase sum drifts from the
    exact sum by up to ~1e-6 turns here; the kernel replays it exactly, so the
    output stays within the f32 bar of the oracle over the whole utterance."""
    rng = np.random.default_rng(7)
    n_mel = 2000
    f0 = f0_contour(rng, 1, n_mel, unvoiced_frac=0.05)
    phase, noise, lw = nsf_inputs(rng, 1, n_mel)
    lw *= 4.0  # amplify phase errors through the merge
    got = run_nsf(ops, f0, 480, phase, noise, lw, 0.0)
    ref = O.nsf_source(f0, 480, phase, noise, lw, 0.0)
    assert_close_f32(got, ref, what="nsf 40 s")
    # and the last second alone agrees to the same bar
    assert_close_f32(got[:, -24000:], ref[:, -24000:], what="nsf last second")


def test_nsf_source_edge_cases(ops):
    rng = np.random.default_rng(8)
    n_mel, up = 24, 480
    f0 = np.zeros((5, n_mel), np.float32)
    f0[1] = 10.0                        # exactly the threshold: unvoiced (f > 10 is voiced)
    f0[2] = np.float32(np.nextafter(np.float32(10.0), np.float32(20.0)))
    f0[3, ::2] = 24000.0 / 3            # high, non-dyadic increments
    f0[4] = 187.5                       # dyadic increments: ties are possible
    phase, noise, lw = nsf_inputs(rng, 5, n_mel, up)
    got = run_nsf(ops, f0, up, phase, noise, lw, -0.02)
    ref = O.nsf_source(f0, up, phase, noise, lw, -0.02)
    assert_close_f32(got, ref, what="nsf edges")
    # silence: only noise at 0.1/3 amplitude
    assert np.all(np.isfinite(got))


def test_nsf_source_other_rates_and_negative_f0(ops):
    rng = np.random.default_rng(9)
    f0 = f0_contour(rng, 2, 12)
    f0[1, 3:6] *= -1.0                   # sign changes: the plain-add path
    phase, noise, lw = nsf_inputs(rng, 2, 12, 256)
    got = run_nsf(ops, f0, 256, phase, noise, lw, 0.1, sr=22050)
    ref = O.nsf_source(f0, 256, phase, noise, lw, 0.1, sampling_rate=22050)
    assert_close_f32(got, ref, what="nsf 22.05 kHz, f0 < 0")


def test_nsf_source_nan_propagates_like_the_engine(ops):
    rng = np.random.default_rng(10)
    f0 = f0_contour(rng, 1, 8)
    f0[0, 4] = np.nan
    phase, noise, lw = nsf_inputs(rng, 1, 8, 64)
    got = run_nsf(ops, f0, 64, phase, noise, lw, 0.0)
    ref = O.nsf_source(f0, 64, phase, noise, lw, 0.0)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert_close_f32(got[fin], ref[fin], what="nsf finite part")


def test_nsf_source_batch_independence(ops):
    """An utterance's source does not depend on its batch neighbours."""
    rng = np.random.default_rng(11)
    f0 = f0_contour(rng, 3, 50)
    phase, noise, lw = nsf_inputs(rng, 3, 50)
    all3 = run_nsf(ops, f0, 480, phase, noise, lw, 0.0)
    one = run_nsf(ops, f0[1:2], 480, phase[1:2], noise[1:2], lw, 0.0)
    assert np.array_equal(all3[1:2], one)


def test_nsf_source_empty_and_bad_arguments(ops):
    from chatterbox_amdvulkan_b200 import _lib
    L = _lib.load()
    assert L.cbx_nsf_source(None, 0, 10, 480, 24000, None, None, None, 0.0, None, None) == 0
    assert L.cbx_nsf_source(None, 2, 10, 0, 24000, None, None, None, 0.0, None, None) == -1
    with pytest.raises(ValueError):
        ops.nsf_source(dev(np.zeros((1, 4), np.float32)), 480, dev(np.zeros((1, 9), np.float32)),
                       dev(np.zeros((1, 9, 10), np.float32)), np.zeros(9, np.float32))


# -------------------------------------------------------------------- STFT --

@pytest.mark.parametrize("n_fft,hop", [(16, 4), (8, 2), (32, 8), (4, 1), (16, 16), (2, 1)])
@pytest.mark.parametrize("layout", ["BTC", "BCT"])
def test_stft_parity(ops, n_fft, hop, layout):
    rng = np.random.default_rng(n_fft * 10 + hop)
    x = (0.3 * rng.standard_normal((3, 2501))).astype(np.float32)
    x[1, 100:140] = 0.0
    win = O.hann_window(n_fft)
    got = host(ops.stft(dev(x), n_fft, hop, dev(win), layout=layout))
    ref = O.stft(x, n_fft, hop, win, layout=O.BTC if layout == "BTC" else O.BCT)
    assert got.shape == ref.shape
    assert_close_f32(got, ref, what=f"stft {n_fft}/{hop} {layout}")


def test_stft_hift_source_length_and_minimal_signal(ops):
    rng = np.random.default_rng(12)
    # 10 s at 24 kHz: 60001 frames
    x = np.tanh(0.2 * rng.standard_normal((2, 240000))).astype(np.float32)
    got = host(ops.stft(dev(x)))
    assert got.shape == (2, 60001, 18)
    pick = np.r_[0:40, 30000:30040, 59960:60001]
    ref = O.stft(x)
    assert_close_f32(got[:, pick], ref[:, pick], what="stft 10 s")
    # T = n_fft / 2 + 1: the smallest signal reflect padding accepts
    x9 = rng.standard_normal((1, 9)).astype(np.float32)
    assert_close_f32(host(ops.stft(dev(x9))), O.stft(x9), what="stft T=9")


def test_stft_is_linear_and_exactly_scalable(ops):
    rng = np.random.default_rng(13)
    x = (0.4 * rng.standard_normal((1, 1000))).astype(np.float32)
    s1 = host(ops.stft(dev(x)))
    s2 = host(ops.stft(dev(2.0 * x)))
    assert np.array_equal(s2, 2.0 * s1)


def test_stft_bad_arguments(ops):
    from chatterbox_amdvulkan_b200 import _lib
    L = _lib.load()
    assert L.cbx_stft(None, 1, 100, 15, 4, None, 1, None, None) == -1   # odd n_fft
    assert L.cbx_stft(None, 1, 100, 64, 4, None, 1, None, None) == -1   # > 32
    assert L.cbx_stft(None, 1, 8, 16, 4, None, 1, None, None) == -1     # T <= n_fft / 2
    assert L.cbx_stft(None, 1, 100, 16, 17, None, 1, None, None) == -1  # hop > n_fft
    assert L.cbx_stft(None, 0, 100, 16, 4, None, 1, None, None) == 0


# ------------------------------------------------------------------- iSTFT --

def _post(rng, B, Tf, nb=9):
    p = np.concatenate([rng.normal(-2.0, 0.9, (B, nb, Tf)), rng.normal(0.0, 2.0, (B, nb, Tf))],
                       axis=1).astype(np.float32)
    if Tf > 9:
        p[:, 0, 3] = 6.0   # exp > 100: magnitude clamp
        p[:, 2, 9] = 30.0
    return p


@pytest.mark.parametrize("limit", [0.99, np.inf])
@pytest.mark.parametrize("layout", ["BTC", "BCT"])
def test_istft_post_parity(ops, layout, limit):
    rng = np.random.default_rng(14)
    p = _post(rng, 3, 5001)
    x = np.ascontiguousarray(p.transpose(0, 2, 1)) if layout == "BTC" else p
    win = O.hann_window(16)
    got = host(ops.istft_post(dev(x), 16, 4, dev(win), layout=layout, audio_limit=limit))
    ref = O.istft_post(x, 16, 4, win, layout=O.BTC if layout == "BTC" else O.BCT,
                       audio_limit=limit)
    assert got.shape == ref.shape == (3, 20000)
    assert_close_f32(got, ref, what=f"istft {layout} limit={limit}")


@pytest.mark.parametrize("n_fft,hop", [(8, 2), (32, 8), (4, 1), (16, 16), (32, 1)])
def test_istft_post_other_sizes(ops, n_fft, hop):
    rng = np.random.default_rng(n_fft + hop)
    nb = n_fft // 2 + 1
    p = _post(rng, 2, 777, nb)
    win = O.hann_window(n_fft)
    got = host(ops.istft_post(dev(p), n_fft, hop, dev(win), layout="BCT", audio_limit=np.inf))
    ref = O.istft_post(p, n_fft, hop, win, layout=O.BCT, audio_limit=np.inf)
    assert_close_f32(got, ref, what=f"istft {n_fft}/{hop}")


def test_istft_post_short_and_empty(ops):
    rng = np.random.default_rng(15)
    p = _post(rng, 1, 2)
    got = host(ops.istft_post(dev(p), layout="BCT"))
    assert got.shape == (1, 4)
    assert_close_f32(got, O.istft_post(p, layout=O.BCT), what="istft 2 frames")
    from chatterbox_amdvulkan_b200 import _lib
    L = _lib.load()
    assert L.cbx_istft_post(None, 1, 1, 16, 4, None, 1, 0.99, None, None) == 0  # no samples
    assert L.cbx_istft_post(None, 1, 10, 16, 4, None, 1, -1.0, None, None) == -1


def test_istft_post_hift_length(ops):
    """10 s of output (60001 frames, B = 4), sampled rows against the oracle."""
    rng = np.random.default_rng(16)
    p = _post(rng, 4, 60001)
    x = np.ascontiguousarray(p.transpose(0, 2, 1))
    got = host(ops.istft_post(dev(x)))
    assert got.shape == (4, 240000)
    ref = O.istft_post(x[1:3])
    assert_close_f32(got[1:3], ref, what="istft 10 s")
    assert np.max(np.abs(got)) <= np.float32(0.99)


# ------------------------------------------- persistent bulk-copy kernels --
# n_fft 16 / hop 4 (the engine's) and 8 / 2 with 16-byte aligned inputs run
# the persistent kernels (bulk async copies, two-stage ring); misaligned inputs
# run the one-tile-per-CTA kernels.  Both must meet the same bar.

def _offset(a, off):
    """Device copy of `a` starting `off` floats into a larger buffer."""
    flat = dev(np.ascontiguousarray(a).reshape(-1))
    buf = torch.zeros(flat.numel() + off, dtype=torch.float32, device="cuda")
    buf[off:] = flat
    return buf[off:].view(a.shape)


@pytest.mark.parametrize("off", [0, 1, 2, 3])
@pytest.mark.parametrize("layout", ["BTC", "BCT"])
def test_istft_aligned_and_misaligned_inputs(ops, layout, off):
    rng = np.random.default_rng(20 + off)
    p = _post(rng, 3, 1999)
    x = np.ascontiguousarray(p.transpose(0, 2, 1)) if layout == "BTC" else p
    win = O.hann_window(16)
    got = host(ops.istft_post(_offset(x, off), 16, 4, dev(win), layout=layout, audio_limit=np.inf))
    ref = O.istft_post(x, 16, 4, win, layout=O.BTC if layout == "BTC" else O.BCT,
                       audio_limit=np.inf)
    assert_close_f32(got, ref, what=f"istft {layout} off={off}")


@pytest.mark.parametrize("off", [0, 1, 3])
@pytest.mark.parametrize("layout", ["BTC", "BCT"])
def test_stft_aligned_and_misaligned_inputs(ops, layout, off):
    rng = np.random.default_rng(30 + off)
    x = (0.3 * rng.standard_normal((3, 4003))).astype(np.float32)
    win = O.hann_window(16)
    got = host(ops.stft(_offset(x, off), 16, 4, dev(win), layout=layout))
    ref = O.stft(x, 16, 4, win, layout=O.BTC if layout == "BTC" else O.BCT)
    assert_close_f32(got, ref, what=f"stft {layout} off={off}")


def test_istft_phase_arguments_over_the_whole_sin_range(ops):
    """The phase node's sin takes the raw conv_post value: large, negative and
    beyond-range arguments (|x| >= 12000 takes sinf), inf and NaN."""
    rng = np.random.default_rng(40)
    p = _post(rng, 2, 600)
    big = np.array([1e-30, -0.5, 3.14159274, -3.14159274, 1.5707964, 100.25, -777.0, 4096.5,
                    -11999.0, 11999.99, 12000.0, -25000.0, 1e6, -3e7], np.float32)
    p[0, 9:, 100:100 + len(big)] = big[None, :]
    p[1, 9:, 200:200 + len(big)] = -big[None, ::-1]
    for layout in ("BTC", "BCT"):
        x = np.ascontiguousarray(p.transpose(0, 2, 1)) if layout == "BTC" else p
        got = host(ops.istft_post(dev(x), layout=layout, audio_limit=np.inf))
        ref = O.istft_post(x, layout=O.BTC if layout == "BTC" else O.BCT, audio_limit=np.inf)
        assert_close_f32(got, ref, what=f"istft large phases {layout}")
    q = p.copy()
    q[0, 10, 50] = np.inf
    q[1, 11, 70] = np.nan
    got = host(ops.istft_post(dev(q), layout="BCT", audio_limit=np.inf))
    ref = O.istft_post(q, layout=O.BCT, audio_limit=np.inf)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert_close_f32(got[fin], ref[fin], what="istft inf / nan phase")


@pytest.mark.parametrize("layout", ["BTC", "BCT"])
def test_dsp_many_tiles_per_cta(ops, layout):
    """24 x 10 s: every CTA of the persistent kernels walks many tiles, so both
    ring stages cycle through many phases."""
    rng = np.random.default_rng(41)
    B, Tf = 24, 60001
    p = _post(rng, B, Tf)
    x = np.ascontiguousarray(p.transpose(0, 2, 1)) if layout == "BTC" else p
    lay = O.BTC if layout == "BTC" else O.BCT
    got = host(ops.istft_post(dev(x), layout=layout))
    assert_close_f32(got, O.istft_post(x, layout=lay), what=f"istft 24 x 10 s {layout}")
    a = np.tanh(0.3 * rng.standard_normal((B, 240000))).astype(np.float32)
    got = host(ops.stft(dev(a), layout=layout))
    assert_close_f32(got, O.stft(a, layout=lay), what=f"stft 24 x 10 s {layout}")


@pytest.mark.parametrize("T", [9, 10, 11, 12, 13, 17, 1020, 1021, 1024, 1028, 1029, 1036, 1037])
def test_stft_tile_boundaries_and_reflection(ops, T):
    """Lengths around one tile (256 frames = 1020 samples of hop): reflect
    padding on both edges of single- and two-tile signals, odd B * T totals
    (the input's last 16 bytes partial)."""
    rng = np.random.default_rng(T)
    for B in (1, 3):
        x = rng.standard_normal((B, T)).astype(np.float32)
        for layout in ("BTC", "BCT"):
            got = host(ops.stft(dev(x), layout=layout))
            ref = O.stft(x, layout=O.BTC if layout == "BTC" else O.BCT)
            assert_close_f32(got, ref, what=f"stft T={T} B={B} {layout}")


@pytest.mark.parametrize("Tf", [2, 3, 4, 5, 6, 252, 253, 254, 255, 256, 257, 258, 505, 506])
def test_istft_tile_boundaries(ops, Tf):
    """Frame counts around one tile (1002 output samples, 256 frames)."""
    rng = np.random.default_rng(Tf)
    for B in (1, 3):
        p = _post(rng, B, Tf)
        for layout in ("BTC", "BCT"):
            x = np.ascontiguousarray(p.transpose(0, 2, 1)) if layout == "BTC" else p
            got = host(ops.istft_post(dev(x), layout=layout, audio_limit=np.inf))
            ref = O.istft_post(x, layout=O.BTC if layout == "BTC" else O.BCT, audio_limit=np.inf)
            assert_close_f32(got, ref, what=f"istft Tf={Tf} B={B} {layout}")
