"""World-size-2 gloo run of the sequence-sharded path (CPU, no GPU).

Each rank takes its share of a lognormal (cfg5-shaped) batch from
partition_by_context, attends its own sequences over its own pool (the CPU
oracle stands in for the device kernels here), and the rows are all-gathered
as the benchmark does; rank 0 checks the reassembly against a single-process
run and the max-over-ranks timing reduction.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rows_for(seqs, ctx, seed):
    """Oracle attention rows of the given sequences (independent per sequence)."""
    import sys
    sys.path.insert(0, ROOT)
    from oracle.attention import CausalMask, flash_attention
    out = []
    for i in seqs:
        rng = np.random.default_rng(seed + i)
        c = int(ctx[i])
        q = rng.standard_normal((1, 8, 1, 16)).astype(np.float32)
        k = rng.standard_normal((1, 2, c, 16)).astype(np.float32)
        v = rng.standard_normal((1, 2, c, 16)).astype(np.float32)
        out.append(flash_attention(q, k, v, CausalMask())[0, :, 0])
    return np.stack(out) if out else np.zeros((0, 8, 16), np.float32)


def _worker(rank, world, port, ctx, result):
    import sys
    sys.path.insert(0, ROOT)
    from chenxing_b200.sharding import (gather_ragged_rows, max_over_ranks,
                                        partition_by_context, sum_over_ranks)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    try:
        groups = partition_by_context(ctx, world)
        mine = groups[rank]
        local = torch.from_numpy(_rows_for(mine, ctx, 100))
        full = gather_ragged_rows(local, [len(g) for g in groups])
        t_max = max_over_ranks(10.0 + rank)
        units = sum_over_ranks(float(ctx[mine].sum()))
        if rank == 0:
            order = [i for g in groups for i in g]
            result.put((full.numpy(), order, t_max, units))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_rows_match_single_process():
    from chenxing_b200.workloads import lognormal_ctx
    ctx = lognormal_ctx(24, seed=2, median=64, cap=300)
    ctxm = mp.get_context("spawn")
    q = ctxm.SimpleQueue()
    port = _free_port()
    procs = [ctxm.Process(target=_worker, args=(r, 2, port, ctx, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    full, order, t_max, units = q.get()
    ref = _rows_for(order, ctx, 100)
    np.testing.assert_allclose(full, ref, rtol=0, atol=0)
    assert sorted(order) == list(range(len(ctx)))
    assert t_max == 11.0 and units == float(ctx.sum())


def _router_worker(rank, world, port, result):
    import sys
    sys.path.insert(0, ROOT)
    from chenxing_b200.sharding import AdmissionRouter, partition_by_context
    from chenxing_b200.workloads import lognormal_ctx
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    try:
        ctx = lognormal_ctx(64, seed=6)
        router = AdmissionRouter(ctx, partition_by_context(ctx, world), 0.05, seed=11)
        stream = iter(lognormal_ctx(4096, seed=12))
        mine = []                       # what this rank would run, step by step
        for _ in range(20):
            fins = router.finish_step()
            placed = router.admit([next(stream) for _ in range(sum(len(f) for f in fins))])
            router.grow()
            mine.append((fins[rank], [sid for sid, r, _ in placed if r == rank],
                         router.live(rank)))
        views = [None] * world
        dist.all_gather_object(views, (rank, router.rank_of, mine))
        if rank == 0:
            result.put(views)
    finally:
        dist.destroy_process_group()


def test_two_ranks_route_admissions_identically_without_messages():
    """Each rank builds its own AdmissionRouter copy; with no message between
    them they agree on every sequence's rank, and each rank's own view of its
    finishes, admissions and live set is the other copy's view of that rank."""
    ctxm = mp.get_context("spawn")
    q = ctxm.SimpleQueue()
    port = _free_port()
    procs = [ctxm.Process(target=_router_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    views = q.get()
    (_, rank_of0, mine0), (_, rank_of1, mine1) = sorted(views, key=lambda v: v[0])
    assert rank_of0 == rank_of1
    for step0, step1 in zip(mine0, mine1):
        live0, live1 = set(step0[2]), set(step1[2])
        assert not live0 & live1
    assert set(mine0[-1][2]) | set(mine1[-1][2]) == set(rank_of0)
    assert all(rank_of0[s] == 0 for s in mine0[-1][2])
    assert all(rank_of0[s] == 1 for s in mine1[-1][2])
