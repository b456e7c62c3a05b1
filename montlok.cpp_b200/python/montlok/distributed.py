"""Row-sharded prediction over the ranks of a torch.distributed group.

Rows are independent, so N ranks (one process per GPU, as torchrun launches
them) split a batch into contiguous slices of ceil(batch / N) rows, each rank
predicts its own slice on its own device, and the slices are gathered in
rank order; nothing crosses ranks except that gather. ``max_over_ranks`` is
the timing reduction a multi-GPU benchmark reports (the slowest rank).

The predict function is the caller's (normally ``Model.predict``), so the
same code runs on NCCL ranks with GPUs and on gloo ranks without.
"""

from __future__ import annotations

from typing import Callable

import numpy as np


def shard(batch: int, rank: int, world: int) -> tuple[int, int]:
    """The rows [lo, hi) rank `rank` of `world` owns: contiguous slices of
    ceil(batch / world) rows, the last ones shorter or empty."""
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError("need 0 <= rank < world and batch >= 0")
    step = -(-batch // world)
    lo = min(batch, rank * step)
    return lo, min(batch, lo + step)


def predict_sharded(predict: Callable[[np.ndarray], np.ndarray], x: np.ndarray, group=None) -> np.ndarray:
    """Every rank passes the same `x`; each predicts its shard of the rows and
    all ranks return the whole [batch, outputs] result, in row order."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    lo, hi = shard(len(x), rank, world)
    part = np.asarray(predict(np.ascontiguousarray(x[lo:hi])))
    parts: list = [None] * world
    dist.all_gather_object(parts, part, group=group)
    parts = [np.asarray(p) for p in parts]
    return np.concatenate([p[:, None] if p.ndim == 1 else p for p in parts], axis=0)


def max_over_ranks(values: list[float], group=None, device=None) -> list[float]:
    """Element-wise maximum of `values` over the ranks (a tensor on `device`:
    the rank's GPU for NCCL, the CPU for gloo)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(v) for v in t.tolist()]
