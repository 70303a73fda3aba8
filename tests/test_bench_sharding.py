"""bench.py's configs[2] workload is one fixed job split across ranks (strong
scaling): the ranks' shards partition the job's rows, every rank draws the
same job ids and slices its own rows out of them, and every rank reports the
job's bytes (the one-GPU figure).  Built on the CPU (no launch is made)."""
import os
import sys

import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


@pytest.fixture(scope="module")
def bench():
    from chatterbox_amdvulkan_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libcbx_ops.so not built")
    import bench as b
    return b


def _make(bench, rank, world, N=4096, H=64):
    return bench.T3PrefillLarge(torch, torch.device("cpu"), 1000 + rank, N=N, H=H, F=4 * H,
                                rank=rank, world=world)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_partition_the_job_and_share_its_bytes(bench, world):
    whole = _make(bench, 0, 1)
    parts = [_make(bench, r, world) for r in range(world)]
    assert sum(p.rows for p in parts) == whole.rows == whole.job_rows
    assert torch.equal(torch.cat([p.ids for p in parts]), whole.ids)
    assert torch.equal(torch.cat([p.pids for p in parts]), whole.pids)
    assert {p.job_bytes_per_step for p in parts} == {whole.job_bytes_per_step}
    assert whole.job_bytes_per_step == whole.bytes_per_step
    # a rank's own bytes shrink with its shard, but each rank reads its own
    # table rows, so the shards' sum is at least the job's
    assert sum(p.bytes_per_step for p in parts) >= whole.job_bytes_per_step
    # the result gather: rank 0's block is a view of the job's output buffer
    y, y_full, counts = parts[0].gather
    assert counts == [p.rows for p in parts]
    assert y_full.shape[0] == whole.rows and y.data_ptr() == y_full.data_ptr()


def test_make_workload_shards_only_the_strong_workload(bench):
    wl = bench.make_workload("t3_prefill_large_bf16", torch, torch.device("cpu"), 7, rank=1,
                             world=4)
    assert wl.strong and wl.rows == 65536 // 4 and wl.job_rows == 65536
    assert bench.WORKLOADS["t3_prefill_large_bf16"][0].strong
    assert not getattr(bench.WORKLOADS["cfm_ops_f32"][0], "strong", False)


@pytest.mark.parametrize("world,batched", [(1, True), (2, True), (4, True), (8, True), (3, False)])
def test_whole_utterance_shards_take_the_batched_gather(bench, world, batched):
    """configs[2]'s 65,536 rows are 64 utterances of 1,024 tokens: a shard of
    whole utterances calls cbx_embed_gather_add_batched (positions from the
    utterance length, no position-id upload); any other shard passes explicit
    position ids to cbx_embed_gather_add.  Built on the CPU, nothing launched."""
    for rank in range(world):
        wl = bench.make_workload("t3_prefill_large_bf16", torch, torch.device("cpu"), 7,
                                 rank=rank, world=world)
        want = "cbx_embed_gather_add_batched" if batched else "cbx_embed_gather_add"
        assert wl.gather_call == want
        ins = wl.chunks[0][0]
        assert len(ins) == (1 if batched else 2)   # the ids (and the position ids)
