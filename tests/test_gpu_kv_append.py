"""GPU parity of cbx_qkv_kv_append (the T3 QKV epilogue with KV-cache writes,
t3.cpp:465-489) against the oracle: bit-exact (one f32 add, one rounding to
the cache type)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from _gpu import dev, host

pytestmark = pytest.mark.gpu

TORCH_OF = {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


def _cache(shape, t, fill=0.0):
    c = torch.full(shape, fill, dtype=torch.float32, device="cuda")
    return c.to(TORCH_OF[t])


def _host_cache(c, t):
    return host(c) if t == O.F32 else host(c).view(np.uint16)


def _oracle_cache(shape, t, fill=0.0):
    a = np.full(shape, fill, np.float32)
    return a if t == O.F32 else O.to_type(a, t).reshape(shape)


@pytest.mark.parametrize("t", [O.F32, O.F16, O.BF16])
def test_prefill_chunk_bit_exact(ops, golden, t):
    """One stream's prefill chunk: rows n_past .. n_past + N - 1 of one slab."""
    g = golden
    D = g["kv_q"].shape[1]
    ck, cv = _cache((16, D), t), _cache((16, D), t)
    q, err = ops.qkv_kv_append(dev(g["kv_h"]), dev(g["kv_b"]), ck, cv, pos_offset=3,
                               max_context=16)
    rk, rv = _oracle_cache((16, D), t), _oracle_cache((16, D), t)
    rq, rerr = O.qkv_kv_append(g["kv_h"], g["kv_b"], rk, rv, t, pos_offset=3, max_context=16)
    assert int(host(err)[0]) == rerr == 0
    assert np.array_equal(host(q), rq)
    assert np.array_equal(_host_cache(ck, t), rk) and np.array_equal(_host_cache(cv, t), rv)
    if t == O.F32:
        assert np.array_equal(host(q), g["kv_q"]) and np.array_equal(host(ck)[3:8], g["kv_k"])


@pytest.mark.parametrize("t", [O.F32, O.F16, O.BF16])
@pytest.mark.parametrize("D", [1024, 100, 6])
def test_batched_decode_step_bit_exact(ops, t, D):
    """One new token per stream, each at its own position in its own slab."""
    rng = np.random.default_rng(D)
    B, ctx = 37, 50
    x = (3.0 * rng.standard_normal((B, 3 * D))).astype(np.float32)
    b = rng.standard_normal(3 * D).astype(np.float32)
    pos = rng.integers(0, ctx, B).astype(np.int32)
    ck, cv = _cache((B, ctx, D), t, 5.0), _cache((B, ctx, D), t, 5.0)
    q, err = ops.qkv_kv_append(dev(x), dev(b), ck, cv, positions=torch.from_numpy(pos).cuda(),
                               slab_stride=ctx * D, max_context=ctx)
    rk, rv = _oracle_cache((B, ctx, D), t, 5.0), _oracle_cache((B, ctx, D), t, 5.0)
    rq, _ = O.qkv_kv_append(x, b, rk, rv, t, positions=pos, slab_stride=ctx * D, max_context=ctx)
    assert int(host(err)[0]) == 0
    assert np.array_equal(host(q), rq)
    assert np.array_equal(_host_cache(ck, t), rk) and np.array_equal(_host_cache(cv, t), rv)


def test_out_of_range_positions_flagged_and_not_written(ops):
    rng = np.random.default_rng(3)
    B, D, ctx = 6, 64, 8
    x = rng.standard_normal((B, 3 * D)).astype(np.float32)
    pos = np.array([0, 7, 8, -1, 3, 1 << 30], np.int32)
    ck, cv = _cache((B, ctx, D), O.F32, 9.0), _cache((B, ctx, D), O.F32, 9.0)
    q, err = ops.qkv_kv_append(dev(x), None, ck, cv, positions=torch.from_numpy(pos).cuda(),
                               slab_stride=ctx * D, max_context=ctx)
    assert int(host(err)[0]) == 2                      # CBX_EFLAG_POS_OOB
    assert np.array_equal(host(q), x[:, :D])            # Q is written for every row
    k = host(ck)
    for r in (2, 3, 5):
        assert np.all(k[r] == 9.0)                      # nothing written for bad rows
    assert np.array_equal(k[1, 7], x[1, D:2 * D])


def test_strided_rows_no_q_and_misaligned(ops):
    rng = np.random.default_rng(5)
    N, D, ctx = 9, 32, 20
    wide = rng.standard_normal((N, 3 * D + 8)).astype(np.float32)   # qkv_row_stride 3D + 8
    b = rng.standard_normal(3 * D).astype(np.float32)
    from chatterbox_amdvulkan_b200 import _lib
    L = _lib.load()
    xw = dev(wide)
    ck, cv = _cache((ctx, D), O.F32), _cache((ctx, D), O.F32)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    bd = dev(b)
    rc = L.cbx_qkv_kv_append(xw.data_ptr(), 3 * D + 8, bd.data_ptr(), N, D, None, 4,
                             ck.data_ptr(), cv.data_ptr(), 0, 0, ctx, None, err.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    rk, rv = _oracle_cache((ctx, D), O.F32), _oracle_cache((ctx, D), O.F32)
    O.qkv_kv_append(np.ascontiguousarray(wide[:, :3 * D]), b, rk, rv, O.F32, pos_offset=4,
                    max_context=ctx, with_q=False)
    torch.cuda.synchronize()
    assert np.array_equal(host(ck), rk) and np.array_equal(host(cv), rv)
    # misaligned qkv (offset by one float): the scalar path, same result
    buf = torch.zeros(N * 3 * D + 1, device="cuda")
    buf[1:] = dev(np.ascontiguousarray(wide[:, :3 * D]).reshape(-1))
    ck2, cv2 = _cache((ctx, D), O.F32), _cache((ctx, D), O.F32)
    q2, _ = ops.qkv_kv_append(buf[1:].view(N, 3 * D), dev(b), ck2, cv2, pos_offset=4,
                              max_context=ctx)
    assert np.array_equal(host(ck2), rk) and np.array_equal(host(cv2), rv)


def test_kv_append_bad_arguments(ops):
    from chatterbox_amdvulkan_b200 import _lib
    L = _lib.load()
    assert L.cbx_qkv_kv_append(None, 0, None, 0, 64, None, 0, None, None, 0, 0, 8, None, None,
                               None) == 0                                     # no rows
    assert L.cbx_qkv_kv_append(None, 10, None, 2, 64, None, 0, None, None, 0, 0, 8, None, None,
                               None) == -1                                    # stride < 3D
    assert L.cbx_qkv_kv_append(None, 0, None, 2, 64, None, 0, None, None, 7, 0, 8, None, None,
                               None) == -2                                    # cache type
