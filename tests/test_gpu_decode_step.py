"""The batched multi-stream T3 decode step (chatterbox_amdvulkan_b200/
decode_step.py): the library-backed step against the same step in plain torch
fp32, eagerly and replayed from one CUDA graph."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dec():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import decode_step
    torch.backends.cuda.matmul.allow_tf32 = False  # the same exact f32 GEMMs in both paths
    return decode_step


def _history(m, seed):
    """Random cache contents for earlier positions (identical in both copies)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    m.cache_k.copy_(torch.randn(m.cache_k.shape, generator=g, device="cuda").to(m.cache_k.dtype))
    m.cache_v.copy_(torch.randn(m.cache_v.shape, generator=g, device="cuda").to(m.cache_v.dtype))
    return m.cache_k.clone(), m.cache_v.clone()


@pytest.mark.parametrize("cache_dtype", [torch.float32, torch.bfloat16])
def test_decode_step_matches_torch_reference(dec, cache_dtype):
    B, ctx = 12, 48
    m = dec.T3BatchedDecode(n_layers=3, B=B, max_context=ctx, cache_dtype=cache_dtype, seed=3)
    rk, rv = _history(m, 4)
    g = torch.Generator(device="cuda").manual_seed(5)
    pos = torch.randint(0, ctx, (B,), generator=g, device="cuda", dtype=torch.int32)
    x = torch.randn(B, m.D, generator=g, device="cuda")
    y = m.step(x, pos)
    yr = m.step_reference(x, pos, rk, rv)
    torch.cuda.synchronize()
    assert int(m.err.item()) == 0
    # the elementwise ops agree to f32 rounding; GEMMs and attention are shared.
    # A bf16 cache rounds K / V to 8 bits: a 1e-7 difference upstream can flip
    # a rounding (one bf16 ulp, 2^-8 relative), which the attention carries on.
    tol, ctol = (2e-5, 2e-5) if cache_dtype == torch.float32 else (2e-3, 2.0 ** -8)
    assert dec.rel_err(y, yr) < tol
    assert dec.rel_err(m.cache_k.float(), rk.float()) < ctol
    assert dec.rel_err(m.cache_v.float(), rv.float()) < ctol


def test_decode_steps_replayed_from_one_cuda_graph(dec):
    """Capture one step; replay it for 4 steps with advancing positions and new
    tokens; the results equal eager steps of a twin model."""
    B, ctx = 16, 40
    m = dec.T3BatchedDecode(n_layers=2, B=B, max_context=ctx, seed=7)
    twin = dec.T3BatchedDecode(n_layers=2, B=B, max_context=ctx, seed=7)
    g = torch.Generator(device="cuda").manual_seed(8)
    pos0 = torch.randint(0, ctx - 5, (B,), generator=g, device="cuda", dtype=torch.int32)
    xs = [torch.randn(B, m.D, generator=g, device="cuda") for _ in range(4)]
    x_static = xs[0].clone()
    pos_static = pos0.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m.step(x_static, pos_static)  # warm-up (cuBLAS handles, workspaces)
    torch.cuda.current_stream().wait_stream(s)
    m.cache_k.zero_()
    m.cache_v.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_static = m.step(x_static, pos_static)
    m.cache_k.zero_()
    m.cache_v.zero_()
    for i, x in enumerate(xs):
        x_static.copy_(x)
        pos_static.copy_(pos0 + i)
        graph.replay()
        y_eager = twin.step(x, pos0 + i)
        torch.cuda.synchronize()
        assert torch.equal(y_static, y_eager), f"step {i}"
    assert torch.equal(m.cache_k, twin.cache_k) and torch.equal(m.cache_v, twin.cache_v)
    del graph


def test_decode_step_flags_positions_past_the_cache(dec):
    B, ctx = 4, 8
    m = dec.T3BatchedDecode(n_layers=1, B=B, max_context=ctx, seed=9)
    pos = torch.tensor([0, 7, 8, 3], dtype=torch.int32, device="cuda")
    m.step(torch.randn(B, m.D, device="cuda"), pos, check=False)
    torch.cuda.synchronize()
    assert int(m.err.item()) == 2  # CBX_EFLAG_POS_OOB: stream 2 has no room left
    assert not m.cache_k[0, 2].any()
    with pytest.raises(dec.PositionOutOfRange):
        m.check_errors()
    assert int(m.err.item()) == 0  # read and cleared


def test_decode_step_raises_on_a_position_equal_to_the_context(dec):
    """An eager step checks the error word itself: a stream at position ==
    max_context raises, and the next in-range step runs clean."""
    B, ctx = 3, 6
    m = dec.T3BatchedDecode(n_layers=2, B=B, max_context=ctx, seed=10)
    x = torch.randn(B, m.D, device="cuda")
    with pytest.raises(dec.PositionOutOfRange):
        m.step(x, torch.tensor([1, ctx, 2], dtype=torch.int32, device="cuda"))
    m.step(x, torch.tensor([1, ctx - 1, 2], dtype=torch.int32, device="cuda"))
    assert int(m.err.item()) == 0
