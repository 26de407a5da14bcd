"""Data parallelism over independent sequences (eight
bs=1 sequences on 1/2/4/8 GPUs).

The sequences share nothing, so each rank decodes its own share with the
single-GPU engine and the only collectives are for bookkeeping: a barrier
around timed regions and max / sum reductions of scalars (the job's time is
the slowest rank's, its token count the sum). One process per GPU; the
process group is NCCL on GPUs and gloo on CPU, and the reductions use a
tensor on the matching device.
"""

from __future__ import annotations

from typing import Sequence, TypeVar

import torch
import torch.distributed as dist

T = TypeVar("T")


def shard(items: Sequence[T], rank: int, world: int) -> list[T]:
    """Round-robin share of `items` for `rank` (rank r gets r, r + world, ...)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    return list(items[rank::world])


def _device() -> torch.device:
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _reduce(x: float, op) -> float:
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=op)
    return float(t.item())


def all_max(x: float, world: int) -> float:
    """Max over ranks (the job time of a data-parallel step)."""
    return x if world == 1 else _reduce(x, dist.ReduceOp.MAX)


def all_sum(x: float, world: int) -> float:
    """Sum over ranks (tokens of a data-parallel step)."""
    return x if world == 1 else _reduce(x, dist.ReduceOp.SUM)


def barrier(world: int) -> None:
    if world > 1:
        dist.barrier()


def gather_lists(values: list, world: int) -> list:
    """Every rank's list, in rank order (host objects)."""
    if world == 1:
        return [values]
    out: list = [None] * world
    dist.all_gather_object(out, values)
    return out
