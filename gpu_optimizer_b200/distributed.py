"""One-process-per-GPU plumbing for sharded candidate evaluation.

Candidate evaluation has no exchange step, so torch.distributed is used
only for control: a barrier around timed regions and max / sum reductions
of host scalars (the slowest rank's time, the total candidate count).
Works with the ``nccl`` backend on GPUs and ``gloo`` on CPU ranks.
"""

from __future__ import annotations

from collections.abc import Sequence

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
