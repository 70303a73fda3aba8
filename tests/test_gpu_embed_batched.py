"""cbx_embed_gather_add_batched: n_batch utterances of seq_len tokens at the
same positions n_past .. n_past + seq_len - 1 (t3.cpp:440-455 per utterance,
positions as t3.cpp:597-600), bit-exact against the CPU oracle's gather with
pos_ids[b * seq_len + t] = n_past + t.  Covers the position-major kernel
(both register widths), the row-kernel fallbacks (mixed types, odd hidden,
wide rows), out-of-range ids and positions, and configs[2]'s full shape."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from _gpu import dev, host

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


def _table(rng, rows, H, t):
    return O.to_type((0.02 * rng.standard_normal((rows, H))).astype(np.float32), t)


def _oracle(tok, tok_t, ids, pos, pos_t, n_past, out_t):
    B, T = ids.shape
    pids = (n_past + np.tile(np.arange(T), B)).astype(np.int32)
    return O.embed_gather_add(tok, tok_t, ids.reshape(-1), pos, pos_t, pos_ids=pids,
                              out_t=out_t)


def _run(ops, tok, tok_t, ids, pos, pos_t, n_past, out_t):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.embed_gather_add_batched(
        dev(tok, tok_t), torch.from_numpy(ids).cuda(),
        None if pos is None else dev(pos, pos_t), n_past,
        out_dtype={O.F32: torch.float32, O.BF16: torch.bfloat16, O.F16: torch.float16}[out_t],
        err_word=err)
    torch.cuda.synchronize()
    return host(out).reshape(ids.shape[0] * ids.shape[1], -1), int(err.item())


@pytest.mark.parametrize("tt,ot", [(O.BF16, O.BF16), (O.F16, O.F16), (O.F32, O.F32),
                                   (O.BF16, O.F32), (O.F16, O.BF16), (O.F32, O.BF16)])
@pytest.mark.parametrize("B,T,H,n_past", [
    (64, 40, 1024, 0),    # configs[2]'s hidden, many utterances per position
    (3, 37, 1024, 5),     # chunks split at position boundaries
    (1, 70, 1024, 0),     # one utterance: one row per position
    (5, 7, 2048, 2),      # 16-bit rows of 256 vectors (wide register path)
    (2, 9, 256, 100),     # short rows
])
def test_batched_bit_exact(ops, tt, ot, B, T, H, n_past):
    rng = np.random.default_rng(B * 1000 + T + H)
    V, P = 6563, 4096
    tok = _table(rng, V, H, tt)
    pos = _table(rng, P, H, tt)
    ids = rng.integers(0, 6561, (B, T)).astype(np.int32)
    ids.reshape(-1)[0], ids.reshape(-1)[-1] = 0, V - 1
    got, err = _run(ops, tok, tt, ids, pos, tt, n_past, ot)
    ref, rf = _oracle(tok, tt, ids, pos, tt, n_past, ot)
    assert err == 0 and rf == 0
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("tt,pt,H", [
    (O.BF16, O.F16, 1024),   # mixed table types: row kernels, positions n_past + r % T
    (O.F32, O.F32, 1001),    # hidden not a whole number of vectors: scalar kernel
    (O.BF16, O.BF16, 4096),  # rows wider than the register path
    (O.F16, O.F16, 3000),    # 16-bit, 375 vectors per row
])
def test_batched_fallbacks_bit_exact(ops, tt, pt, H):
    rng = np.random.default_rng(H)
    B, T, n_past = 4, 33, 7
    tok = _table(rng, 500, H, tt)
    pos = _table(rng, 64, H, pt)
    ids = rng.integers(0, 500, (B, T)).astype(np.int32)
    got, err = _run(ops, tok, tt, ids, pos, pt, n_past, O.F32)
    ref, rf = _oracle(tok, tt, ids, pos, pt, n_past, O.F32)
    assert err == 0 and rf == 0
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("tt", [O.BF16, O.F32])
def test_batched_out_of_range(ops, tt):
    """Bad ids and positions past the table: zero rows and both flags, as
    cbx_embed_gather_add; the valid rows are unchanged."""
    rng = np.random.default_rng(5)
    B, T, H, V, P, n_past = 6, 20, 1024, 300, 30, 15   # positions 30..34 are past the table
    tok = _table(rng, V, H, tt)
    pos = _table(rng, P, H, tt)
    ids = rng.integers(0, V, (B, T)).astype(np.int32)
    ids[1, 3], ids[4, 0], ids[5, 19] = -1, V, 1 << 30
    got, err = _run(ops, tok, tt, ids, pos, tt, n_past, O.F32)
    ref, rf = _oracle(tok, tt, ids, pos, tt, n_past, O.F32)
    assert rf == err == (O.EFLAG_TOKEN_OOB | O.EFLAG_POS_OOB)
    assert np.array_equal(got, ref)
    rows = got.reshape(B, T, H)
    assert not rows[1, 3].any() and not rows[4, 0].any() and not rows[:, T - 1].any()


def test_batched_no_position_table(ops):
    rng = np.random.default_rng(8)
    tok = _table(rng, 900, 1024, O.BF16)
    ids = rng.integers(0, 900, (7, 50)).astype(np.int32)
    got, err = _run(ops, tok, O.BF16, ids, None, O.BF16, 0, O.BF16)
    ref, rf = O.embed_gather_add(tok, O.BF16, ids.reshape(-1), out_t=O.BF16)
    assert err == 0 and rf == 0
    assert np.array_equal(got, ref)


def test_batched_many_groups_per_warp(ops):
    """262,144 rows of 256 elements: every warp walks several groups of 32 rows
    whose position changes inside a group."""
    rng = np.random.default_rng(9)
    B, T, H = 48, 5461, 256
    tok = _table(rng, 6563, H, O.F16)
    pos = _table(rng, 8192, H, O.F16)
    ids = rng.integers(0, 6563, (B, T)).astype(np.int32)
    got, err = _run(ops, tok, O.F16, ids, pos, O.F16, 3, O.F16)
    ref, rf = _oracle(tok, O.F16, ids, pos, O.F16, 3, O.F16)
    assert err == 0 and rf == 0
    assert np.array_equal(got, ref)


def test_batched_config2_equals_row_gather(ops):
    """configs[2] at full size (64 x 1024 rows, bf16): the batched call equals
    cbx_embed_gather_add with explicit position ids, bit for bit, and a sample
    of rows equals the oracle."""
    g = torch.Generator(device="cuda").manual_seed(1000)
    H, V, P = 1024, 6563, 4096
    tok = (0.02 * torch.randn((V, H), generator=g, device="cuda")).to(torch.bfloat16)
    pos = (0.02 * torch.randn((P, H), generator=g, device="cuda")).to(torch.bfloat16)
    ids = torch.randint(0, 6561, (64, 1024), generator=g, device="cuda", dtype=torch.int32)
    pids = (torch.arange(65536, device="cuda", dtype=torch.int32) % 1024)
    a = ops.embed_gather_add_batched(tok, ids, pos, 0, out_dtype=torch.bfloat16)
    b = ops.embed_gather_add(tok, ids.reshape(-1), pos, pos_ids=pids, out_dtype=torch.bfloat16)
    assert torch.equal(a.reshape(65536, H).view(torch.int16), b.view(torch.int16))
    pick = np.random.default_rng(0).choice(65536, 512, replace=False)
    ref, rf = O.embed_gather_add(host(tok), O.BF16, ids.reshape(-1).cpu().numpy()[pick],
                                 host(pos), O.BF16, pos_ids=(pick % 1024).astype(np.int32),
                                 out_t=O.BF16)
    assert rf == 0 and np.array_equal(host(a).reshape(65536, H)[pick], ref)


def test_batched_wrapper_rejects_bad_shapes(ops):
    tok = torch.zeros((10, 64), device="cuda")
    with pytest.raises(ValueError):
        ops.embed_gather_add_batched(tok, torch.zeros(12, dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        ops.embed_gather_add_batched(tok, torch.zeros((2, 3), dtype=torch.int32, device="cuda"),
                                     out=torch.empty(5, device="cuda"))


def test_batched_empty(ops):
    tok = torch.zeros((10, 64), device="cuda")
    out = ops.embed_gather_add_batched(tok, torch.zeros((0, 7), dtype=torch.int32, device="cuda"))
    assert tuple(out.shape) == (0, 7, 64)
    out = ops.embed_gather_add_batched(tok, torch.zeros((3, 0), dtype=torch.int32, device="cuda"))
    assert tuple(out.shape) == (3, 0, 64)
