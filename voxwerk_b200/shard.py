"""Multi-GPU host logic: rows are independent (TalkerGenerator.cs:366-385 keeps no state across rows; every
sequence owns its history and its Random, :304 and :345-346), so a batch splits into contiguous row shards, one per
rank, and each rank samples its shard with no collective on the data path.  torch.distributed carries only the
start barrier, the max-over-ranks of the device timings, and (when a caller wants one rank to hold every id) the
gather of the ids.
"""

from __future__ import annotations

from typing import List

import numpy as np


def shard_bounds(costs: List[float], rank: int, world: int) -> List[tuple]:
    """(segment, lo, hi) row ranges of `rank`'s contiguous shard, balancing the summed per-row cost.

    `costs[s]` is the list of per-row costs of segment s flattened as (n_rows, cost_per_row); the shard of rank r
    covers cost [total * r / world, total * (r + 1) / world), rounded to whole rows, so consecutive ranks meet
    exactly and the union is the whole batch.
    """
    total = sum(n * c for n, c in costs)
    lo_c, hi_c = total * rank / world, total * (rank + 1) / world
    out, acc = [], 0.0
    for s, (n, per) in enumerate(costs):
        seg_lo = acc
        a = min(n, int(round(max(0.0, lo_c - seg_lo) / per))) if per else 0
        b = min(n, int(round(max(0.0, min(hi_c, seg_lo + per * n) - seg_lo) / per))) if per else 0
        if b > a:
            out.append((s, a, b))
        acc = seg_lo + per * n
    return out


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over every rank of the default process group (itself when not distributed)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    """The sum of `value` over every rank of the default process group (itself when not distributed)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_ids(local_ids: np.ndarray, device=None) -> np.ndarray:
    """Every rank's ids concatenated in rank order (ranks may hold different row counts)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return np.asarray(local_ids, dtype=np.int32)
    world = dist.get_world_size()
    n = torch.tensor([int(local_ids.size)], dtype=torch.int64, device=device)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n)
    counts = [int(c.item()) for c in counts]
    width = max(max(counts), 1)
    buf = torch.full((width,), -1, dtype=torch.int32, device=device)
    buf[: local_ids.size] = torch.from_numpy(np.ascontiguousarray(local_ids, dtype=np.int32)).to(buf.device)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    return np.concatenate([p[:c].cpu().numpy() for p, c in zip(parts, counts)])
