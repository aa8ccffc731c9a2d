"""Request sharding across GPUs (one process per GPU).

The draft-tree cycle has no cross-request data flow: every request's score,
build, verify and commit is independent, so requests are partitioned over
ranks and each rank runs `DraftTreeCycle` on its own shard with its own state
pool; the n-gram table and layer weights are replicated.  There is no
collective on the data path.  `torch.distributed` is used only outside it:
a barrier, the max over ranks of a device time, and gathering per-request
results for a scheduler on rank 0.

The reference plugin is batch-1 per worker (fc1_branch64.py:13); this module
is the host-side layer that maps a global request batch onto ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int     # first global request index of this rank
    count: int     # requests on this rank

    @property
    def stop(self) -> int:
        return self.start + self.count

    def global_ids(self) -> range:
        return range(self.start, self.stop)


def partition(n_requests: int, world: int) -> list[Shard]:
    """Contiguous balanced split: the first n % world ranks get one more."""
    if world <= 0 or n_requests < 0:
        raise ValueError("world must be positive and n_requests non-negative")
    base, extra = divmod(n_requests, world)
    out, start = [], 0
    for r in range(world):
        c = base + (1 if r < extra else 0)
        out.append(Shard(r, world, start, c))
        start += c
    return out


def local_shard(n_requests: int, rank: int | None = None, world: int | None = None) -> Shard:
    """This rank's shard (rank / world from the process group when omitted)."""
    if rank is None:
        rank = dist.get_rank() if dist.is_initialized() else 0
    if world is None:
        world = dist.get_world_size() if dist.is_initialized() else 1
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return partition(n_requests, world)[rank]


def owner_of(request: int, n_requests: int, world: int) -> int:
    """Rank that owns global request index `request`."""
    if not 0 <= request < n_requests:
        raise IndexError(request)
    for s in partition(n_requests, world):
        if s.start <= request < s.stop:
            return s.rank
    raise AssertionError("unreachable")


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (device times are reported as the slowest rank's)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(local: torch.Tensor, n_requests: int, device=None) -> torch.Tensor | None:
    """Concatenate per-rank [count, ...] results in global request order on rank 0
    (None on other ranks).  Outside the timed region: a scheduler's read-back."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    world, rank = dist.get_world_size(), dist.get_rank()
    shards = partition(n_requests, world)
    if local.shape[0] != shards[rank].count:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard has {shards[rank].count}")
    width = max(s.count for s in shards)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=device or local.device)
    pad[: local.shape[0]] = local.to(pad.device)
    parts = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, parts, dst=0)
    if rank != 0:
        return None
    return torch.cat([p[: s.count] for p, s in zip(parts, shards)], 0)
