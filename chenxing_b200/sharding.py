"""Sequence sharding across the GPUs of one node.

Requests are independent, so a multi-GPU run gives each rank its own block
pool and radix subtree and a disjoint set of sequences; the data path has no
collective.  ``partition_by_context`` balances ranks by KV tokens (longest
processing time first), which matters for lognormal context mixes.
``gather_rows`` is the one collective: an all-gather of per-step attention
outputs used when the caller needs every rank's rows (benchmarking the
partitioned path).
"""
from __future__ import annotations

import heapq

import numpy as np

__all__ = ["partition_by_context", "gather_rows", "gather_ragged_rows", "max_over_ranks",
           "sum_over_ranks"]


def partition_by_context(ctx_lens, world: int) -> list[list[int]]:
    """Split sequence indices into ``world`` groups with near-equal token sums.

    Deterministic: longest first, ties to the lowest index, each sequence to
    the currently lightest rank (ties to the lowest rank); indices inside a
    group stay ascending."""
    ctx = np.asarray(ctx_lens, dtype=np.int64)
    order = sorted(range(len(ctx)), key=lambda i: (-int(ctx[i]), i))
    heap = [(0, r) for r in range(world)]
    groups: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        groups[r].append(i)
        heapq.heappush(heap, (load + int(ctx[i]), r))
    return [sorted(g) for g in groups]


def gather_rows(local, group=None):
    """All-gather equally shaped per-rank tensors into one (world * n, ...) tensor."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def gather_ragged_rows(local, n_rows_per_rank, group=None):
    """All-gather per-rank row blocks of different lengths: pads each rank's
    block to the longest, gathers, and strips the padding (rank order)."""
    import torch
    pad = max(n_rows_per_rank)
    buf = torch.zeros((pad,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    full = gather_rows(buf, group)
    return torch.cat([full[r * pad:r * pad + n] for r, n in enumerate(n_rows_per_rank)])


def _reduce(value: float, op, device, group=None) -> float:
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op, group=group)
    return float(t.item())


def max_over_ranks(value: float, device="cpu", group=None) -> float:
    """Step time of a multi-GPU run: the slowest rank's device time."""
    import torch.distributed as dist
    return _reduce(value, dist.ReduceOp.MAX, device, group)


def sum_over_ranks(value: float, device="cpu", group=None) -> float:
    import torch.distributed as dist
    return _reduce(value, dist.ReduceOp.SUM, device, group)
