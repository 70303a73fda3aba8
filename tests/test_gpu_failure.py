"""Failure detection on the GPU without a fault: a bounded wait that runs out
(an mbarrier nothing completes) must raise the device error word, the host
must read CBX_ERR_TIMEOUT, the word must clear, and the context must stay
usable."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import _lib
    return _lib.load()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_bounded_wait_times_out_and_reports(lib):
    flags = ctypes.c_int32(-1)
    assert lib.cbx_device_errors(ctypes.byref(flags), _stream()) == 0 and flags.value == 0
    assert lib.cbx_selftest_wait_timeout(1000, _stream()) == 0
    rc = lib.cbx_device_errors(ctypes.byref(flags), _stream())
    assert rc == -5 and flags.value == 1          # CBX_ERR_TIMEOUT, CBX_DEVERR_WAIT_TIMEOUT
    assert b"0x1" in lib.cbx_last_error()
    assert lib.cbx_device_errors(ctypes.byref(flags), _stream()) == 0 and flags.value == 0


def test_context_usable_after_timeout(lib):
    from chatterbox_amdvulkan_b200 import ops
    import oracle as O
    assert lib.cbx_selftest_wait_timeout(100, _stream()) == 0
    x = np.linspace(-5, 5, 4096, dtype=np.float32)
    y = ops.gelu(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.allclose(y, O.gelu_tanh(x), rtol=1e-5, atol=1e-6)
    flags = ctypes.c_int32(0)
    assert lib.cbx_device_errors(ctypes.byref(flags), _stream()) == -5


def test_selftest_rejects_bad_limits(lib):
    assert lib.cbx_selftest_wait_timeout(0, _stream()) == -1
    assert lib.cbx_selftest_wait_timeout((1 << 24) + 1, _stream()) == -1
