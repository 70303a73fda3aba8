"""The T3 prefill input sequence through cbx_t3_embed_sequence (t3.cpp:428-455):
[cond rows ; speech_emb[prompt] ; tok_table[tokens]] + pos_embd[n_past + i],
bit-exact against the CPU oracle and the reference's own fixture, at the
engine's table shapes (text table 50276 x 1024 in f16, as the GGUF ships it)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle as O
from _gpu import dev, host

pytestmark = pytest.mark.gpu

H, TEXT_V, SPEECH_V, CTX = 1024, 50276, 6563, 8196


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from chatterbox_amdvulkan_b200 import ops as _ops
    return _ops


@pytest.fixture(scope="module")
def tables():
    """The engine's three tables in f16 (host storage + device copies)."""
    rng = np.random.default_rng(11)
    t = {}
    for name, rows in (("text", TEXT_V), ("speech", SPEECH_V), ("pos", CTX)):
        a = (0.02 * rng.standard_normal((rows, H))).astype(np.float16)
        t[name] = (a.view(np.uint16), dev(a.view(np.uint16), O.F16))
    return t


def _ids(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()


def test_sequence_matches_reference_fixture(ops, golden):
    g = golden
    out = ops.t3_embed_sequence(dev(g["seq_text16"], O.F16), _ids(g["seq_text_ids"]),
                                dev(g["seq_pos16"], O.F16), 0, cond=dev(g["seq_cond"]),
                                prompt_table=dev(g["seq_speech16"], O.F16),
                                prompt_ids=_ids(g["seq_prompt_ids"]))
    assert np.array_equal(host(out), g["seq_y"])


@pytest.mark.parametrize("n_prompt,n_text,n_past,cond", [
    (150, 80, 0, True),      # the engine's prefill: speaker row, prompt, text
    (0, 57, 0, True),        # no prompt speech
    (0, 200, 0, False),      # text only (t3.cpp:284)
    (33, 1, 0, True),        # one text token
    (1, 0, 12, True),        # speech prompt only (no text rows)
    (0, 0, 5, True),         # the conditioning row alone
    (300, 500, 1000, True),  # a later chunk (n_past > 0)
])
def test_sequence_engine_shapes_bit_exact(ops, tables, n_prompt, n_text, n_past, cond):
    rng = np.random.default_rng(n_prompt * 7 + n_text + n_past)
    c = rng.standard_normal(H).astype(np.float32) if cond else None
    pi = rng.integers(0, SPEECH_V, n_prompt).astype(np.int32)
    ti = rng.integers(0, TEXT_V, n_text).astype(np.int32)
    # the ids at the tables' edges
    if n_text >= 2:
        ti[0], ti[-1] = 0, TEXT_V - 1
    if n_prompt >= 2:
        pi[0], pi[-1] = SPEECH_V - 1, 0
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.t3_embed_sequence(tables["text"][1], _ids(ti), tables["pos"][1], n_past,
                                cond=None if c is None else dev(c),
                                prompt_table=tables["speech"][1] if n_prompt else None,
                                prompt_ids=_ids(pi) if n_prompt else None, err_word=err)
    ref, rf = O.t3_embed_sequence(tables["text"][0], O.F16, ti, tables["pos"][0], O.F16, n_past,
                                  c, tables["speech"][0], O.F16, pi if n_prompt else None)
    assert rf == 0 and int(err.item()) == 0
    assert np.array_equal(host(out), ref)


@pytest.mark.parametrize("out_t", [O.F32, O.BF16, O.F16])
def test_sequence_batch_of_utterances_large(ops, tables, out_t):
    """65,536 rows in one call: a speaker row, a 1000-row prompt and 64,535
    text rows drawn over the whole 50,276-row table (103 MB in f16: not
    L2-resident), against a 65,600-row position table; every output type;
    checked in full, with no flag raised."""
    rng = np.random.default_rng(5)
    c = rng.standard_normal(H).astype(np.float32)
    pi = rng.integers(0, SPEECH_V, 1000).astype(np.int32)
    ti = rng.integers(0, TEXT_V, 65536 - 1001).astype(np.int32)
    big_pos = (0.02 * rng.standard_normal((65600, H))).astype(np.float16).view(np.uint16)
    tdt = {O.F32: torch.float32, O.BF16: torch.bfloat16, O.F16: torch.float16}[out_t]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.t3_embed_sequence(tables["text"][1], _ids(ti), dev(big_pos, O.F16), 50,
                                cond=dev(c), prompt_table=tables["speech"][1],
                                prompt_ids=_ids(pi), out_dtype=tdt, err_word=err)
    ref, rf = O.t3_embed_sequence(tables["text"][0], O.F16, ti, big_pos, O.F16, 50, c,
                                  tables["speech"][0], O.F16, pi, out_t=out_t)
    assert rf == 0 and int(err.item()) == 0
    assert np.array_equal(host(out), ref)


def test_sequence_out_of_range_ids_and_positions(ops, tables):
    """A bad id in either segment, and positions past the table: zero rows and
    the flags, no out-of-range read; the other rows are untouched."""
    rng = np.random.default_rng(3)
    c = rng.standard_normal(H).astype(np.float32)
    pi = rng.integers(0, SPEECH_V, 20).astype(np.int32)
    ti = rng.integers(0, TEXT_V, 30).astype(np.int32)
    pi[4], ti[7], ti[8] = SPEECH_V, -1, TEXT_V
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    n_past = CTX - 45       # the last 6 rows fall past the position table
    out = ops.t3_embed_sequence(tables["text"][1], _ids(ti), tables["pos"][1], n_past,
                                cond=dev(c), prompt_table=tables["speech"][1],
                                prompt_ids=_ids(pi), err_word=err)
    ref, rf = O.t3_embed_sequence(tables["text"][0], O.F16, ti, tables["pos"][0], O.F16, n_past,
                                  c, tables["speech"][0], O.F16, pi)
    assert rf == (O.EFLAG_TOKEN_OOB | O.EFLAG_POS_OOB) == int(err.item())
    got = host(out)
    assert np.array_equal(got, ref)
    assert not got[1 + 4].any() and not got[21 + 7].any() and not got[-1].any()


def test_sequence_mixed_types_and_misaligned_tables(ops, tables):
    """bf16 prompt table with f16 text / positions, and a misaligned text
    table (the scalar kernel), against the oracle."""
    rng = np.random.default_rng(9)
    sp32 = (0.02 * rng.standard_normal((SPEECH_V, H))).astype(np.float32)
    sp_bf = O.to_type(sp32, O.BF16)
    pi = rng.integers(0, SPEECH_V, 40).astype(np.int32)
    ti = rng.integers(0, TEXT_V, 70).astype(np.int32)
    c = rng.standard_normal(H).astype(np.float32)
    out = ops.t3_embed_sequence(tables["text"][1], _ids(ti), tables["pos"][1], 3, cond=dev(c),
                                prompt_table=dev(sp_bf, O.BF16), prompt_ids=_ids(pi))
    ref, _ = O.t3_embed_sequence(tables["text"][0], O.F16, ti, tables["pos"][0], O.F16, 3, c,
                                 sp_bf, O.BF16, pi)
    assert np.array_equal(host(out), ref)
    # hidden 1023 over buffers that start one element in: not 16-byte vectors
    Hm = H - 1
    flat = tables["text"][1].reshape(-1)[1: 1 + 5000 * Hm].view(5000, Hm)
    pos_m = tables["pos"][1].reshape(-1)[1: 1 + 300 * Hm].view(300, Hm)
    tim = rng.integers(0, 5000, 64).astype(np.int32)
    out = ops.t3_embed_sequence(flat, _ids(tim), pos_m, 0)
    flat_h = tables["text"][0].reshape(-1)[1: 1 + 5000 * Hm].reshape(5000, Hm)
    pos_h = tables["pos"][0].reshape(-1)[1: 1 + 300 * Hm].reshape(300, Hm)
    ref, _ = O.t3_embed_sequence(flat_h, O.F16, tim, pos_h, O.F16, 0)
    assert np.array_equal(host(out), ref)


# ---------------------------------------------------------------- batched --

def _batched(ops, tables, B, n_prompt, n_text, n_past, n_cond, seed, out_dtype=torch.float32,
             prompt_table=None, prompt_host=None, prompt_t=O.F16):
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((B, n_cond, H)).astype(np.float32) if n_cond else None
    pi = rng.integers(0, SPEECH_V, (B, n_prompt)).astype(np.int32)
    ti = rng.integers(0, TEXT_V, (B, n_text)).astype(np.int32)
    sp_d = tables["speech"][1] if prompt_table is None else prompt_table
    sp_h = tables["speech"][0] if prompt_host is None else prompt_host
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.t3_embed_sequence_batched(tables["text"][1], _ids(ti), tables["pos"][1], n_past,
                                        cond=None if c is None else dev(c),
                                        prompt_table=sp_d if n_prompt else None,
                                        prompt_ids=_ids(pi) if n_prompt else None,
                                        out_dtype=out_dtype, err_word=err)
    got = host(out)
    out_t = {torch.float32: O.F32, torch.bfloat16: O.BF16, torch.float16: O.F16}[out_dtype]
    flags = 0
    for b in range(B):
        ref, rf = O.t3_embed_sequence(tables["text"][0], O.F16, ti[b], tables["pos"][0], O.F16,
                                      n_past, None if c is None else c[b], sp_h, prompt_t,
                                      pi[b] if n_prompt else None, out_t=out_t)
        flags |= rf
        assert np.array_equal(got[b], ref), f"utterance {b}"
    return got, flags, int(err.item())


@pytest.mark.parametrize("B,n_prompt,n_text,n_past,n_cond", [
    (64, 150, 873, 0, 1),    # the bench's batch: speaker row, prompt, text per utterance
    (3, 0, 57, 0, 1),        # no prompt speech
    (5, 0, 200, 0, 0),       # text only
    (2, 33, 1, 7, 1),        # one text token
    (4, 12, 0, 12, 1),       # prompt only
    (6, 0, 0, 5, 2),         # conditioning rows alone, two per utterance
    (300, 4, 9, 900, 1),     # more utterances than resident CTAs
])
def test_sequence_batched_bit_exact(ops, tables, B, n_prompt, n_text, n_past, n_cond):
    _, flags, err = _batched(ops, tables, B, n_prompt, n_text, n_past, n_cond,
                             seed=B + n_prompt + n_text)
    assert flags == err == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_sequence_batched_output_types(ops, tables, out_dtype):
    _, flags, err = _batched(ops, tables, 8, 40, 300, 3, 1, seed=21, out_dtype=out_dtype)
    assert flags == err == 0


def test_sequence_batched_mixed_types(ops, tables):
    """A bf16 prompt table with f16 text / positions takes the scalar kernel,
    one grid row per utterance."""
    rng = np.random.default_rng(31)
    sp_bf = O.to_type((0.02 * rng.standard_normal((SPEECH_V, H))).astype(np.float32), O.BF16)
    _, flags, err = _batched(ops, tables, 5, 20, 60, 0, 1, seed=32,
                             prompt_table=dev(sp_bf, O.BF16), prompt_host=sp_bf,
                             prompt_t=O.BF16)
    assert flags == err == 0


def test_sequence_batched_out_of_range(ops, tables):
    """Positions past the table in every utterance (n_past near the end): the
    same zero rows and flag as the single-utterance call."""
    got, flags, err = _batched(ops, tables, 3, 10, 20, CTX - 25, 1, seed=41)
    assert flags == err == O.EFLAG_POS_OOB
    assert not got[:, -1].any()


def test_sequence_batched_wrapper_rejects_bad_shapes(ops, tables):
    ids = torch.zeros((2, 5), dtype=torch.int32, device="cuda")
    with pytest.raises(TypeError):
        ops.t3_embed_sequence_batched(tables["text"][1], ids.reshape(-1))
    with pytest.raises(ValueError):
        ops.t3_embed_sequence_batched(tables["text"][1], ids,
                                      prompt_table=tables["speech"][1],
                                      prompt_ids=torch.zeros((3, 2), dtype=torch.int32,
                                                             device="cuda"))


def test_sequence_batched_empty_batch(ops, tables):
    """No utterances: an empty result and no launch."""
    ids = torch.zeros((0, 5), dtype=torch.int32, device="cuda")
    out = ops.t3_embed_sequence_batched(tables["text"][1], ids, tables["pos"][1], 0,
                                        cond=torch.zeros((0, H), device="cuda"))
    assert tuple(out.shape) == (0, 5, H)
