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


def gather_rows(local: torch.Tensor, counts: list[int] | None = None) -> torch.Tensor | None:
    """Gather each rank's row block to rank 0 in rank order (the final result
    gather).  Blocks may differ in their first dimension (uneven shards): they
    are padded to the largest block for the collective and trimmed after.
    Returns the concatenated tensor on rank 0, None on the other ranks."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world, rank = dist.get_world_size(), dist.get_rank()
    if counts is None:
        n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
        all_n = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(all_n, n)
        counts = [int(c.item()) for c in all_n]
    top = max(counts)
    padded = local
    if local.shape[0] < top:
        padded = torch.zeros((top,) + tuple(local.shape[1:]), dtype=local.dtype,
                             device=local.device)
        padded[: local.shape[0]] = local
    buf = torch.empty((world * top,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(buf, padded.contiguous())
    if rank != 0:
        return None
    return torch.cat([buf[r * top: r * top + counts[r]] for r in range(world)])
