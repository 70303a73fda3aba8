"""Shared pytest configuration: the `gpu` marker and common fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "ref_ops.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


def assert_close_f32(got, ref, atol=1e-6, rtol=1e-5, what=""):
    """fp32 parity bar: |got - ref| <= atol + rtol * |ref| elementwise; NaN must match NaN."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_g, nan_r = np.isnan(got), np.isnan(ref)
    assert np.array_equal(nan_g, nan_r), f"{what}: NaN pattern differs"
    ok = ~nan_r
    inf_r = np.isinf(ref) & ok
    assert np.array_equal(got[inf_r], ref[inf_r]), f"{what}: Inf differs"
    fin = ok & ~inf_r
    err = np.abs(got[fin] - ref[fin])
    bound = atol + rtol * np.abs(ref[fin])
    if err.size:
        i = int(np.argmax(err / bound))
        assert np.all(err <= bound), (
            f"{what}: max err/bound {float((err / bound)[i]):.3f} at flat {i}: "
            f"got {got[fin][i]!r} ref {ref[fin][i]!r}")


def bf16_ulp(v):
    """Spacing of bf16 numbers at |v| (v as float64 array)."""
    v = np.abs(np.asarray(v, np.float64))
    e = np.floor(np.log2(np.maximum(v, 2.0 ** -126)))
    return 2.0 ** (e - 7)


def assert_within_bf16_ulps(got_f32, ref_f32, ulps=2, what="", atol=1e-6):
    """bf16 parity bar: got (bf16 widened to f32) within `ulps` bf16 ulp of the
    f32 oracle result rounded to bf16, with the f32 bar's absolute floor of
    1e-6 (values that cancel to ~1e-7 carry f32 rounding noise of ~1e-8, many
    bf16 ulp at that magnitude)."""
    import oracle as O
    ref_b = O.to_f32(O.to_type(np.asarray(ref_f32, np.float32), O.BF16), O.BF16)
    got = np.asarray(got_f32, np.float64)
    ref = np.asarray(ref_b, np.float64)
    assert np.array_equal(np.isnan(got), np.isnan(ref)), f"{what}: NaN pattern differs"
    fin = np.isfinite(ref)
    err = np.abs(got[fin] - ref[fin])
    bound = ulps * bf16_ulp(ref[fin]) + atol
    if err.size:
        i = int(np.argmax(err / bound))
        assert np.all(err <= bound), (
            f"{what}: err/bound {float((err / bound)[i]):.2f} ({ulps} bf16 ulp + {atol}) at {i}: "
            f"got {got[fin][i]!r} ref {ref[fin][i]!r}")
