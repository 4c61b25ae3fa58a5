"""One-process-per-GPU plumbing for partitioned candidate evaluation.

Candidate evaluation has no exchange step, so NCCL is not used: a ``gloo``
process group on host tensors carries the control traffic -- a barrier
around timed regions, max / sum reductions of host scalars (the slowest
rank's time, the total candidate count), the gather of result objects --
and the group's key-value store hands out work.

``pull_partition`` is the partition of one search batch over the ranks
(the per-batch loop of optimizer/search/loop.py:138-172 spread over
devices): every rank takes the next unclaimed candidate from a counter in
the store (an atomic ``add``), so a rank that drew slow candidates takes
fewer of them, and the results come back to every rank in proposal order.
"""

from __future__ import annotations

import time
from collections.abc import Callable, Sequence

import torch
import torch.distributed as dist


def _active() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def shard(items: Sequence, rank: int, world_size: int) -> list:
    """Round-robin shard of a proposal batch; rank r gets items r, r+W, ..."""
    return list(items[rank::world_size])


def unshard(parts: Sequence[Sequence], n: int) -> list:
    """Inverse of ``shard``: per-rank result lists back to proposal order."""
    out = [None] * n
    w = len(parts)
    for r, part in enumerate(parts):
        for j, v in enumerate(part):
            out[r + j * w] = v
    return out


def _device() -> torch.device:
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def reduce_scalar(x: float, op: str = "max") -> float:
    """Max or sum of a host scalar over all ranks (identity without a group)."""
    if not _active():
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier() -> None:
    if _active():
        dist.barrier()


def gather_objects(obj) -> list:
    """All ranks' objects, in rank order (host pickles; control data only)."""
    if not _active():
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


_batches = 0  # batches partitioned so far; equal on every rank


def pull_partition(items: Sequence, evaluate: Callable, order: Sequence[int] | None = None,
                   ) -> tuple[list, dict]:
    """Evaluate ``items`` across all ranks; every rank gets all results.

    ``order`` is the dispatch order (indices into ``items``; default the
    proposal order): a longest-first order lets the ranks finish together.
    Results are returned in proposal order, with per-rank statistics:
    ``busy_s`` (seconds spent in ``evaluate``), ``count`` and ``wall_s``
    (from the common start to the rank's last result).
    Every rank must call this with the same items in the same sequence.
    """
    global _batches
    _batches += 1
    n = len(items)
    order = list(range(n)) if order is None else list(order)
    if sorted(order) != list(range(n)):
        raise ValueError("order must be a permutation of the item indices")
    rank, size = world()
    key = f"gpo_pull_partition/{_batches}"
    store = dist.distributed_c10d._get_default_store() if _active() else None
    local: list = []
    busy = 0.0
    barrier()
    t0 = time.perf_counter()
    taken = 0
    while True:
        if store is not None:
            i = int(store.add(key, 1)) - 1
        else:
            i = taken
        taken += 1
        if i >= n:
            break
        idx = order[i]
        ts = time.perf_counter()
        local.append((idx, evaluate(items[idx])))
        busy += time.perf_counter() - ts
    wall = time.perf_counter() - t0
    stats = {"rank": rank, "busy_s": busy, "count": len(local), "wall_s": wall}
    parts = gather_objects((local, stats))
    out: list = [None] * n
    for part, _ in parts:
        for idx, res in part:
            out[idx] = res
    return out, {"ranks": [s for _, s in parts]}
