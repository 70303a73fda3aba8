"""Row / utterance sharding across GPUs of one node, and the result gather.

Every op of libcbx_ops is independent per row (T3 tokens, CFM (b, t) columns,
Snake (b, c) rows), so a multi-GPU run splits the rows (or the batch of
utterances) into contiguous per-rank blocks and runs the same kernels on each
GPU with no communication.  The only collective is the final gather of the
outputs to rank 0 (NCCL over NVLink/NVSwitch), outside the per-layer path.

Process model: one process per GPU (torchrun), rank r drives cuda:LOCAL_RANK.
Waits on the host are bounded (``wait_event``) so a stuck peer surfaces as an
error instead of a hang.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist


class ShardTimeout(RuntimeError):
    """A bounded wait on the host gave up (maps to CBX_ERR_TIMEOUT)."""


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def shard_range(n: int, world: int, rank: int) -> Shard:
    """Contiguous block of n units for `rank` of `world`: every rank gets
    n // world units and the last n % world ranks one more."""
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, rem = divmod(n, world)
    first_big = world - rem
    start = rank * base + max(0, rank - first_big)
    size = base + (1 if rank >= first_big else 0)
    return Shard(rank, world, start, start + size)


def env_rank() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment (1 process: 0, 0, 1)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: str = "nccl", timeout_s: float = 120.0):
    """Initialise the process group if running under torchrun; returns (rank, local, world)."""
    rank, local, world = env_rank()
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        import datetime
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    elif backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, local, world


def wait_event(event: torch.cuda.Event, timeout_s: float, poll_s: float = 1e-4) -> None:
    """Poll a CUDA event until it completes or `timeout_s` passes (then ShardTimeout)."""
    deadline = time.monotonic() + timeout_s
    while not event.query():
        if time.monotonic() > deadline:
            raise ShardTimeout(f"event not complete after {timeout_s:.3f} s")
        time.sleep(poll_s)


def max_over_ranks(x: float, device=None) -> float:
    """Max of a host scalar over all ranks (the scalar itself when not distributed)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    dev = device if device is not None else (
        torch.device("cuda", torch.cuda.current_device())
        if dist.get_backend() == "nccl" else torch.device("cpu"))
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard_counts(n: int, world: int) -> list[int]:
    """Rows of every rank under shard_range (rank order)."""
    return [shard_range(n, world, r).size for r in range(world)]


def gather_rows_into(local: torch.Tensor, out: torch.Tensor | None,
                     counts: list[int]) -> None:
    """Gather each rank's row block into `out` on rank 0, in rank order (the
    final result gather).  `counts[r]` = rows of rank r; `out` is rank 0's
    preallocated [sum(counts), ...] buffer (ignored elsewhere).  Rank 0 copies
    its own block unless `local` already is out's first block (a view: no
    copy), and receives the others point to point; every other rank sends its
    block once.  So each block crosses the link once, to rank 0 only.
    Enqueued on the current stream (NCCL) and complete when it is."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        if out is not None and out.data_ptr() != local.data_ptr():
            out[: local.shape[0]].copy_(local)
        return
    world, rank = dist.get_world_size(), dist.get_rank()
    if len(counts) != world or local.shape[0] != counts[rank]:
        raise ValueError(f"rank {rank}: {local.shape[0]} rows, counts {counts}")
    if rank != 0:
        if counts[rank]:
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, local.contiguous(), 0)]):
                w.wait()
        return
    if out is None or out.shape[0] != sum(counts) or out.shape[1:] != local.shape[1:]:
        raise ValueError("rank 0 needs an output buffer of sum(counts) rows")
    if counts[0] and out.data_ptr() != local.data_ptr():
        out[: counts[0]].copy_(local)
    ops, start = [], counts[0]
    for r in range(1, world):
        if counts[r]:
            ops.append(dist.P2POp(dist.irecv, out[start: start + counts[r]], r))
        start += counts[r]
    for w in dist.batch_isend_irecv(ops) if ops else []:
        w.wait()


def gather_rows(local: torch.Tensor, counts: list[int] | None = None) -> torch.Tensor | None:
    """Gather each rank's row block to rank 0 in rank order (blocks may differ
    in their first dimension).  Returns the concatenated tensor on rank 0 and
    None on the other ranks; a convenience over gather_rows_into that
    allocates the output and, without `counts`, exchanges the block sizes."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world, rank = dist.get_world_size(), dist.get_rank()
    if counts is None:
        dev = local.device if dist.get_backend() == "nccl" else torch.device("cpu")
        n = torch.tensor([local.shape[0]], dtype=torch.int64, device=dev)
        all_n = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(all_n, n)
        counts = [int(c.item()) for c in all_n]
    out = None
    if rank == 0:
        out = torch.empty((sum(counts),) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
    gather_rows_into(local, out, counts)
    return out
