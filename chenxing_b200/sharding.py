"""Sequence sharding across the GPUs of one node.

Requests are independent, so a multi-GPU run gives each rank its own block
pool and radix subtree and a disjoint set of sequences; the data path has no
collective.  ``partition_by_context`` balances ranks by KV tokens (longest
processing time first), which matters for lognormal context mixes.
``AdmissionRouter`` keeps them balanced under churn: every rank holds an
identical copy and applies the same calls, so all ranks agree on which
sequences finish and where each new request goes without exchanging a
message.  ``gather_rows`` is the one collective: an all-gather of per-step
attention outputs used when the caller needs every rank's rows
(benchmarking the partitioned path).
"""
from __future__ import annotations

import heapq

import numpy as np

__all__ = ["partition_by_context", "deal_by_context", "AdmissionRouter", "gather_rows",
           "gather_ragged_rows", "max_over_ranks", "sum_over_ranks"]


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


def deal_by_context(ctx_lens, world: int) -> list[list[int]]:
    """Split sequence indices into ``world`` groups of equal size (the count
    must divide evenly) with near-equal token sums: longest first (ties to
    the lowest index), dealt round by round in snake order (ranks 0..world-1,
    then world-1..0, ...), so within every round each rank takes one sequence
    and the sums differ by at most the largest length gap of a round.
    Indices inside a group stay ascending."""
    ctx = np.asarray(ctx_lens, dtype=np.int64)
    if world <= 0 or len(ctx) % world:
        raise ValueError("deal_by_context needs a sequence count divisible by world")
    order = sorted(range(len(ctx)), key=lambda i: (-int(ctx[i]), i))
    groups: list[list[int]] = [[] for _ in range(world)]
    for k, i in enumerate(order):
        rnd, pos = divmod(k, world)
        groups[pos if rnd % 2 == 0 else world - 1 - pos].append(i)
    return [sorted(g) for g in groups]


class AdmissionRouter:
    """Churn and admission for sequence-sharded serving, replicated on every rank.

    Tracks each live sequence's rank and KV length.  ``finish_step`` picks the
    sequences that finish this step (``frac`` of each rank's live set, at
    least one, drawn from a generator every copy seeds identically);
    ``admit`` places new requests, longest first, each on the rank with the
    fewest live KV tokens (ties to the lowest rank) -- the rule
    ``partition_by_context`` uses for the initial split; ``grow`` adds the
    tokens each live sequence gained in a step.  Copies built from the same
    arguments and given the same calls make the same decisions, so the ranks
    of a multi-GPU run need no messages to agree.  Sequence ids: the indices
    of ``ctx_lens`` for the initial population, then ``len(ctx_lens)``, ...
    in admission order."""

    def __init__(self, ctx_lens, groups, frac: float, seed: int) -> None:
        self.world = len(groups)
        self.frac = float(frac)
        self._rng = np.random.default_rng(seed)
        self.rank_of: dict = {}
        self.ctx: dict = {}
        self.load = [0] * self.world
        self._live: list[set] = [set() for _ in range(self.world)]
        for r, g in enumerate(groups):
            for i in g:
                self._add(int(i), r, int(ctx_lens[i]))
        self.next_id = len(ctx_lens)

    def _add(self, sid: int, rank: int, n: int) -> None:
        self.rank_of[sid] = rank
        self.ctx[sid] = n
        self.load[rank] += n
        self._live[rank].add(sid)

    def live(self, rank: int) -> list[int]:
        return sorted(self._live[rank])

    def finish_step(self) -> list[list[int]]:
        """Per rank, the ids of the sequences that finish now (removed)."""
        out = []
        for r in range(self.world):
            live = self.live(r)
            if not live:
                out.append([])
                continue
            n = min(len(live), max(1, int(round(self.frac * len(live)))))
            done = sorted(int(x) for x in self._rng.choice(live, size=n, replace=False))
            for sid in done:
                self.load[r] -= self.ctx.pop(sid)
                del self.rank_of[sid]
                self._live[r].discard(sid)
            out.append(done)
        return out

    def admit(self, ctx_lens) -> list[tuple[int, int, int]]:
        """Place new requests; returns (id, rank, context length) in arrival order."""
        ids = list(range(self.next_id, self.next_id + len(ctx_lens)))
        self.next_id += len(ctx_lens)
        order = sorted(range(len(ctx_lens)), key=lambda i: (-int(ctx_lens[i]), i))
        placed = {}
        for i in order:
            r = min(range(self.world), key=lambda k: (self.load[k], k))
            self._add(ids[i], r, int(ctx_lens[i]))
            placed[i] = r
        return [(ids[i], placed[i], int(ctx_lens[i])) for i in range(len(ctx_lens))]

    def grow(self, n: int = 1) -> None:
        """Every live sequence gained ``n`` tokens (one decode step: n = 1)."""
        for r in range(self.world):
            for sid in self._live[r]:
                self.ctx[sid] += n
            self.load[r] += n * len(self._live[r])


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
