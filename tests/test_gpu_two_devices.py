"""One process, two GPUs: the library's per-device state (the shared-memory
opt-in of the kernels that need more than 48 KB, the device error word's
address, occupancy and SM counts) is set up on each device on first use, so
entry points work on whichever device is current, alternating between them.
Skipped unless two GPUs are visible."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from conftest import assert_close_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


def _on(dev, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{dev}")


def test_entry_points_alternate_between_devices(ops):
    from chatterbox_amdvulkan_b200 import _lib
    rng = np.random.default_rng(0)
    B, C, T = 2, 256, 64
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    cb = rng.standard_normal(C).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    tail_ref = O.causal_block1d_tail(x, cb, g, None, 1e-5, None)
    ln_ref = O.layernorm_channels(x, g, None, 1e-5, None, O.BCT, O.ACT_MISH)
    post = np.concatenate([rng.normal(-2.0, 0.9, (B, 600, 9)), rng.normal(0, 2.0, (B, 600, 9))],
                          axis=2).astype(np.float32)
    istft_ref = O.istft_post(post)
    f0 = np.where(rng.random((B, 20)) < 0.2, 0.0, rng.uniform(80, 300, (B, 20))).astype(np.float32)
    phase = rng.uniform(-3, 3, (B, 9)).astype(np.float32)
    noise = rng.standard_normal((B, 9, 20 * 480)).astype(np.float32)
    lw = (0.4 * rng.standard_normal(9)).astype(np.float32)
    nsf_ref = O.nsf_source(f0, 480, phase, noise, lw, 0.01)
    for dev in (0, 1, 0, 1):
        with torch.cuda.device(dev):
            y = ops.causal_block1d_tail(_on(dev, x), _on(dev, cb), _on(dev, g), None, 1e-5)
            assert_close_f32(y.cpu().numpy(), tail_ref, what=f"tail on cuda:{dev}")
            y = ops.layernorm_channels(_on(dev, x), _on(dev, g), None, 1e-5)
            assert_close_f32(y.cpu().numpy(), ln_ref, what=f"ln over C on cuda:{dev}")
            y = ops.istft_post(_on(dev, post))
            assert_close_f32(y.cpu().numpy(), istft_ref, what=f"istft on cuda:{dev}")
            y = ops.nsf_source(_on(dev, f0), 480, _on(dev, phase), _on(dev, noise), lw, 0.01)
            assert_close_f32(y.cpu().numpy(), nsf_ref, what=f"nsf on cuda:{dev}")
            flags = ctypes.c_int32(-1)
            _lib.call("cbx_device_errors", ctypes.byref(flags),
                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert flags.value == 0


def test_wrappers_follow_the_tensor_device_without_a_guard(ops):
    """The torch wrappers make the first tensor's device current for the call,
    so a tensor on cuda:1 works while cuda:0 is current, and a call whose
    tensors sit on two devices is refused before any launch."""
    rng = np.random.default_rng(1)
    B, C, T = 2, 256, 48
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    ref = O.layernorm_channels(x, g, None, 1e-5, None, O.BCT, O.ACT_MISH)
    u = rng.standard_normal(4096).astype(np.float32)
    torch.cuda.set_device(0)
    for dev in (1, 0, 1):
        y = ops.layernorm_channels(_on(dev, x), _on(dev, g), None, 1e-5)
        assert y.device.index == dev and torch.cuda.current_device() == 0
        assert_close_f32(y.cpu().numpy(), ref, what=f"ln over C on cuda:{dev}, cuda:0 current")
        assert_close_f32(ops.gelu(_on(dev, u)).cpu().numpy(), O.gelu_tanh(u),
                         what=f"gelu on cuda:{dev}")
    with pytest.raises(ValueError, match="share its device"):
        ops.layernorm_channels(_on(1, x), _on(0, g), None, 1e-5)


def test_batched_gathers_alternate_between_devices(ops):
    """The batched gather and the batched prefill sequence size their grids
    from the current device's occupancy: alternating devices gives bit-exact
    rows on each."""
    rng = np.random.default_rng(2)
    V, P, H, B, T = 500, 64, 256, 6, 40
    tok = (0.02 * rng.standard_normal((V, H))).astype(np.float32)
    pos = (0.02 * rng.standard_normal((P, H))).astype(np.float32)
    ids = rng.integers(0, V, (B, T)).astype(np.int32)
    pids = (3 + np.tile(np.arange(T), B)).astype(np.int32)
    ref, _ = O.embed_gather_add(tok, O.F32, ids.reshape(-1), pos, O.F32, pos_ids=pids)
    cond = rng.standard_normal((B, 1, H)).astype(np.float32)
    seq_ref = [O.t3_embed_sequence(tok, O.F32, ids[b], pos, O.F32, 3, cond[b])[0]
               for b in range(B)]
    for dev in (1, 0, 1):
        with torch.cuda.device(dev):
            got = ops.embed_gather_add_batched(_on(dev, tok), _on(dev, ids), _on(dev, pos), 3)
            assert np.array_equal(got.reshape(B * T, H).cpu().numpy(), ref)
            seq = ops.t3_embed_sequence_batched(_on(dev, tok), _on(dev, ids), _on(dev, pos), 3,
                                                cond=_on(dev, cond))
            assert np.array_equal(seq.cpu().numpy(), np.stack(seq_ref))
