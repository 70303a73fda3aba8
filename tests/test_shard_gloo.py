"""Multi-rank host logic on CPU: shard partitioning, the result gather to rank 0,
max-over-ranks timing, and failure detection (a rank that never joins, a
bounded wait that runs out) — world_size 2 over gloo, no GPU."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from chatterbox_amdvulkan_b200.shard import ShardTimeout, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (7, 3), (2, 4), (0, 2),
                                     (65536, 8), (100, 7)])
def test_shard_range_partitions_exactly(n, world):
    shards = [shard_range(n, world, r) for r in range(world)]
    assert shards[0].start == 0 and shards[-1].stop == n
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    sizes = [s.size for s in shards]
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n
    assert sizes == sorted(sizes)  # the remainder goes to the last ranks


def test_shard_range_rejects_bad_input():
    with pytest.raises(ValueError):
        shard_range(10, 0, 0)
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _worker(rank, world, port, n_rows, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        from chatterbox_amdvulkan_b200 import shard
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
        sh = shard.shard_range(n_rows, world, rank)
        # each rank "computes" its rows: row i holds value i in every column
        local = torch.arange(sh.start, sh.stop, dtype=torch.float32)[:, None].repeat(1, 3)
        full = shard.gather_rows(local)
        # the preallocated form, rank 0's block a view of the output (no copy)
        counts = shard.shard_counts(n_rows, world)
        out = torch.full((n_rows, 3), -1.0) if rank == 0 else None
        mine = out[: counts[0]] if rank == 0 else local.clone()
        if rank == 0:
            mine.copy_(local)
        shard.gather_rows_into(mine, out, counts)
        t = shard.max_over_ranks(0.5 + rank)
        if rank == 0:
            assert torch.equal(out, full)
            q.put(("ok", full.tolist(), t))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put(("err", repr(e), rank))


@pytest.mark.parametrize("n_rows", [10, 7, 1])
def test_gather_rows_and_max_over_two_gloo_ranks(n_rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_rows, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, full, t = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", full
    assert [row[0] for row in full] == list(range(n_rows))
    assert t == 1.5


def _lonely_worker(port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    t0 = time.monotonic()
    try:
        # world of 2, but rank 1 never joins: the rendezvous must time out
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        q.put(("joined", time.monotonic() - t0))
    except Exception as e:
        q.put(("timeout", time.monotonic() - t0, type(e).__name__))


def test_missing_rank_times_out_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(_free_port(), q))
    p.start()
    res = q.get(timeout=120)
    p.join(timeout=30)
    if p.is_alive():
        p.kill()
    assert res[0] == "timeout", res
    assert res[1] < 60


class _NeverDone:
    def query(self):
        return False


def test_bounded_event_wait_gives_up():
    from chatterbox_amdvulkan_b200.shard import wait_event
    t0 = time.monotonic()
    with pytest.raises(ShardTimeout):
        wait_event(_NeverDone(), timeout_s=0.2)
    assert time.monotonic() - t0 < 5
