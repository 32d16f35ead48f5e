"""GPU parity at the full sizes of the verify, prefix-sharing and churn
workloads (cfg4, cfg3, cfg5).

At these sizes the oracle checks sampled sequences (every sequence's rows
would take minutes in NumPy) and the rest is covered by size-independent
properties: host metadata (block tables, lengths, free lists) bit-exact
against the oracle's replay of the same operations, pool bytes bit-exact
where a kernel copies or must not touch them, every output finite.
Tolerance for bf16 pools: max |out - ref| <= 2e-2 * max |ref| per sequence.
"""
import math

import numpy as np
import pytest
import torch

from gpu_cases import (BF16_RTOL, assert_close_rows, bf16_round, claim_blocks, oracle_rows,
                       pool_rows)

pytestmark = pytest.mark.gpu

HQ, HK, D, BS = 32, 8, 128, 16


@pytest.fixture(autouse=True)
def _clean_flags():
    from chenxing_b200 import _lib
    _lib.device_flags(clear=True)
    yield
    flags = _lib.device_flags(clear=True)
    assert flags == 0, f"device error flags raised: {_lib.describe_flags(flags)}"


def _randn(shape, g, scale=1.0 / math.sqrt(D)):
    return (torch.randn(shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


# ---------------------------------------------------------------------------
# cfg4: speculative verify at full size, then rollback and re-verify
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("gamma", [4, 8])
def test_cfg4_full_size_verify_rollback_reverify(gamma):
    """B 128, ctx ~ U[2048, 16384], gamma + 1 queries per sequence, causal
    within the draft, window 4096, Hq 32 / Hkv 8, D 128, bf16 pool.

    The first verify pass appends and verifies the gamma + 1 chain at [ctx, ctx + gamma].
    The reference then keeps ``a = gamma - rejected`` drafts plus the next
    token and shrinks ``n_tokens`` to ``ctx + a + 1`` without touching the
    table (speculative.py:86-92, 176-184).  The second pass grows the table like
    LLMEngine._ensure_capacity (engine.py:74-85), overwrites the stale slots
    with a new chain at [n', n' + gamma] and verifies again.
    """
    from chenxing_b200 import PagedBatch, RadixPagedKVCache, slot_mapping
    from chenxing_b200.seqmeta import grow_table, rollback
    from chenxing_b200.workloads import verify_meta
    from oracle.paged import ensure_capacity, rollback as o_rollback
    from oracle.radix_kv import OraclePagedKVCache

    seed, W, B = 11 + gamma, 4096, 128
    ctx = np.random.default_rng(seed).integers(2048, 16385, size=B)
    need = int(sum(-(-(int(c) + 2 * gamma + 1) // BS) for c in ctx))
    n_blocks = need + 512
    wl = verify_meta(n_blocks, seed=seed, batch=B, gamma=gamma, window=W)
    assert np.array_equal(wl.ctx_lens, ctx)
    tables = [list(t) for t in wl.block_tables]
    rejected = wl.extra["rejected"]

    cache = RadixPagedKVCache(n_blocks, BS, 1, HK, D, dtype="bfloat16", host_io=False)
    meta = OraclePagedKVCache(n_blocks, BS, 1, HK, D, with_pool=False)
    used = [b for t in tables for b in t]
    claim_blocks(cache, used)
    claim_blocks(meta, used)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    cache._k.normal_(0.0, 1.0 / math.sqrt(D), generator=g)
    cache._v.normal_(0.0, 1.0 / math.sqrt(D), generator=g)
    T = gamma + 1
    sample = sorted({int(np.argmin(ctx)), int(np.argmax(ctx)), 5, 64, 127})

    def verify_round(n_past):
        k_new, v_new = _randn((B * T, HK, D), g), _randn((B * T, HK, D), g)
        q = _randn((B * T, HQ, D), g)
        slots = slot_mapping(tables, n_past, [T] * B, BS)
        cache.append_batch(0, k_new, v_new, slots)
        batch = PagedBatch(cache, tables, n_past + T, n_q_heads=HQ, q_lens=[T] * B, window=W)
        out = cache.verify_batch(0, q, batch).cpu().numpy()
        assert np.isfinite(out).all()
        qh = q.float().cpu().numpy()
        for b in sample:
            lo = max(0, int(n_past[b]) - W + 1)
            kb, vb = pool_rows(cache, 0, tables[b], lo, int(n_past[b]) + T)
            ref = oracle_rows(qh[b * T:(b + 1) * T], kb, vb, window=W)
            # the cfg4 shape at full size: half the bound at most
            assert assert_close_rows(out[b * T:(b + 1) * T], ref, BF16_RTOL, f"seq {b}") <= 0.5
        return k_new, batch

    # ---- first speculative verify step
    k1, batch1 = verify_round(ctx.astype(np.int64))
    assert batch1.kv_tokens == int(sum(min(int(c) + T, W + gamma) for c in ctx))

    # ---- rollback: tables untouched, lengths as the reference computes them
    n_tok = ctx + T
    accepted = gamma - rejected
    target = ctx + accepted + 1
    n_new = np.array([rollback(int(n), int(t)) for n, t in zip(n_tok, target)])
    n_ref = np.array([o_rollback(int(n), int(t)) for n, t in zip(n_tok, target)])
    assert np.array_equal(n_new, n_ref)
    tables_before = [list(t) for t in tables]

    # ---- second verify step: capacity growth bit-exact with the oracle, stale slots overwritten
    o_tables = [list(t) for t in tables]
    for b in range(B):
        grow_table(cache, tables[b], int(n_new[b]) + T)
        ensure_capacity(meta, o_tables[b], int(n_new[b]) + T)
    assert tables == o_tables
    assert cache.free_blocks == meta.free_blocks
    for b in range(B):
        assert tables[b][:len(tables_before[b])] == tables_before[b]
    # the accepted part of the first pass's chain, [ctx, n'), keeps its bytes
    keep = {b: (int(ctx[b]), int(n_new[b])) for b in sample}
    before = {b: pool_rows(cache, 0, tables[b], *keep[b]) for b in sample}
    verify_round(n_new)
    for b, (kb, vb) in before.items():
        ka, va = pool_rows(cache, 0, tables[b], *keep[b])
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)


# ---------------------------------------------------------------------------
# cfg3: radix prefix sharing with a shared partial tail (copy-on-write)
# ---------------------------------------------------------------------------
def _counter_clock():
    import itertools
    c = itertools.count()
    return lambda: float(next(c))


def test_cfg3_full_size_prefix_share_cow_decode():
    """256 requests in 4 groups; each group shares a 2048 + r_g token prefix
    (128 whole blocks through the radix tree, refcount 64, plus a partially
    filled tail block aliased by the group), Hkv 32, D 128, bf16, 2 layers.
    Each request privatises the tail (copy-on-write fused into the suffix
    append), appends its suffix ~ U[128, 512] and one decode token, then
    decodes.  The radix side is the reference's match_prefix / insert /
    acquire (radix_kv.py:150-211), replayed on the oracle in lockstep."""
    from chenxing_b200 import PagedBatch, RadixPagedKVCache, slot_mapping
    from chenxing_b200.seqmeta import grow_table
    from chenxing_b200.workloads import prefix_share_meta
    from oracle.paged import ensure_capacity
    from oracle.radix_kv import OraclePagedKVCache

    hk, hq, L = 32, 32, 2
    meta_w = prefix_share_meta(seed=3)
    P0, tails, suffix = meta_w["prefix_tokens"], meta_w["tail"], meta_w["suffix"]
    G, R = suffix.shape
    n_blocks = G * (P0 // BS + 1) + int(sum(-(-(int(t) + int(s) + 1) // BS) + 1
                                            for t, srow in zip(tails, suffix) for s in srow)) + 64
    cache = RadixPagedKVCache(n_blocks, BS, L, hk, D, dtype="bfloat16", host_io=False,
                              clock=_counter_clock())
    meta = OraclePagedKVCache(n_blocks, BS, L, hk, D, with_pool=False, clock=_counter_clock())
    rng = np.random.default_rng(3)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)

    # ---- writers: one prefix per group, whole blocks published in the tree
    prefix_tok, prefix_kv, gtables = [], [], []
    for gi in range(G):
        plen = P0 + int(tails[gi])
        toks = [100000 * (gi + 1)] + [int(x) for x in rng.integers(0, 50000, size=plen - 1)]
        t, ot = [], []
        grow_table(cache, t, plen)
        ensure_capacity(meta, ot, plen)
        assert t == ot
        kv = _randn((2, L, plen, hk, D), g)
        sl = slot_mapping([t], [0], [plen], BS)
        for l in range(L):
            cache.append_batch(l, kv[0, l], kv[1, l], sl)
        cache.insert(toks[:P0], t[:P0 // BS])
        meta.insert(toks[:P0], ot[:P0 // BS])
        prefix_tok.append(toks)
        prefix_kv.append(kv)
        gtables.append(t)

    # ---- requests: zero-copy prefix hit + aliased tail, then CoW + growth
    tables, otables, n_past, cow = [], [], [], ([], [], [])
    for gi in range(G):
        tail_id = gtables[gi][P0 // BS]
        for ri in range(R):
            prompt = prefix_tok[gi] + [int(x) for x in rng.integers(0, 50000, size=int(suffix[gi, ri]))]
            hit, ohit = cache.match_prefix(prompt), meta.match_prefix(prompt)
            assert hit.n_tokens == ohit.n_tokens == P0
            assert hit.block_ids == ohit.block_ids == gtables[gi][:P0 // BS]
            cache.acquire(hit.node)
            meta.acquire(ohit.node)
            t, ot = hit.block_ids + [tail_id], ohit.block_ids + [tail_id]
            n0 = P0 + int(tails[gi])
            dst, odst = cache.alloc_block(), meta.alloc_block()      # copy-on-write target
            assert dst == odst
            cow[0].append(tail_id)
            cow[1].append(dst)
            cow[2].append(int(tails[gi]))
            t[P0 // BS] = dst
            ot[P0 // BS] = odst
            total = n0 + int(suffix[gi, ri]) + 1
            grow_table(cache, t, total)
            ensure_capacity(meta, ot, total)
            tables.append(t)
            otables.append(ot)
            n_past.append(n0)
    assert tables == otables
    assert cache.free_blocks == meta.free_blocks
    node = cache.match_prefix(prefix_tok[0]).node
    assert node.refcnt == R

    # ---- suffix append with the fused CoW, then one decode token each
    n_past = np.asarray(n_past, dtype=np.int64)
    n_suf = suffix.reshape(-1).astype(np.int64)
    Bn = len(tables)
    suf_kv = _randn((2, L, int(n_suf.sum()), hk, D), g)
    dec_kv = _randn((2, L, Bn, hk, D), g)
    q = _randn((L, Bn, hq, D), g)
    s1 = slot_mapping(tables, n_past, n_suf, BS)
    s2 = slot_mapping(tables, n_past + n_suf, [1] * Bn, BS)
    cow_t = tuple(np.asarray(c, dtype=np.int32) for c in cow)
    batch = PagedBatch(cache, tables, n_past + n_suf + 1, n_q_heads=hq)
    outs = []
    for l in range(L):
        cache.append_batch(l, suf_kv[0, l], suf_kv[1, l], s1, cow=cow_t)
        cache.append_batch(l, dec_kv[0, l], dec_kv[1, l], s2)
        outs.append(cache.decode_batch(l, q[l], batch).cpu().numpy())
    for o in outs:
        assert np.isfinite(o).all()

    # ---- shared blocks untouched; CoW targets hold the tail's valid slots
    for gi in range(G):
        plen = P0 + int(tails[gi])
        for l in range(L):
            kp, vp = pool_rows(cache, l, gtables[gi], 0, plen)
            assert np.array_equal(kp, prefix_kv[gi][0, l].float().cpu().numpy())
            assert np.array_equal(vp, prefix_kv[gi][1, l].float().cpu().numpy())
    starts = np.concatenate([[0], np.cumsum(n_suf)])
    sample = [gi * R + ri for gi in range(G) for ri in (0, R - 1)]
    for b in sample:
        gi = b // R
        plen = P0 + int(tails[gi])
        for l in range(L):
            kb, vb = pool_rows(cache, l, tables[b], 0, plen + int(n_suf[b]) + 1)
            ksrc = torch.cat([prefix_kv[gi][0, l], suf_kv[0, l, starts[b]:starts[b + 1]],
                              dec_kv[0, l, b:b + 1]]).float().cpu().numpy()
            vsrc = torch.cat([prefix_kv[gi][1, l], suf_kv[1, l, starts[b]:starts[b + 1]],
                              dec_kv[1, l, b:b + 1]]).float().cpu().numpy()
            assert np.array_equal(kb, ksrc) and np.array_equal(vb, vsrc), f"request {b} layer {l}"
            ref = oracle_rows(q[l, b:b + 1].float().cpu().numpy(), ksrc, vsrc)
            assert_close_rows(outs[l][b:b + 1], ref, BF16_RTOL, f"request {b} layer {l}")


# ---------------------------------------------------------------------------
# cfg5: continuous-batching churn on one rank's share, through the engine
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("publish_mode", ["suffix", "reference"])
def test_cfg5_rank_share_churn_evict_compact_decode(publish_mode):
    """One rank's share (partition_by_context over 8 ranks) of 1024 sequences
    with lognormal contexts (median 2048, sigma 1.0, cap 32768), Hq 32 /
    Hkv 8, D 128, bf16.  Per step: 5 % finish (prefix published, private
    blocks freed), as many are admitted with a 50 % chance of a 1024-token
    radix hit, LRU eviction plus compaction, then one batched decode step.
    Metadata is compared with the oracle engine replay after every step;
    pool contents with a device-side shadow of every sequence's K/V
    (bit-exact); decode rows of sampled sequences with the oracle.

    ``publish_mode="reference"`` publishes as the reference does (the whole
    chain from token 0 under the hit node).  Evicting such a node frees blocks
    that live sequences still use; at this size and seed no eviction does so,
    which the test asserts before trusting the pool comparison.  In that
    mode the finishing sequences are drawn from those admitted without a radix
    hit: a finished hit sequence's duplicate chain would be the first LRU
    victim and free its hit prefix under the live sequences (the reference
    hazard, shown on the host by test_host_cpu)."""
    from chenxing_b200 import RadixPagedKVCache
    from chenxing_b200.engine import BatchedKVEngine
    from chenxing_b200.sharding import partition_by_context
    from chenxing_b200.workloads import lognormal_ctx
    from engine_replay import OracleEngine
    from oracle.radix_kv import OraclePagedKVCache
    from replay import tree_sig

    ctx_all = lognormal_ctx(1024, seed=5)
    share = partition_by_context(ctx_all, 8)[0]
    rng = np.random.default_rng(5)
    new_ctx = iter(lognormal_ctx(256, seed=55))
    n_blocks = int(1.08 * sum(-(-int(ctx_all[i] + 8) // BS) for i in share)) + 4 * 64
    clock_a, clock_b = _counter_clock(), _counter_clock()
    cache = RadixPagedKVCache(n_blocks, BS, 1, HK, D, dtype="bfloat16", host_io=False,
                              clock=clock_a)
    meta = OraclePagedKVCache(n_blocks, BS, 1, HK, D, with_pool=False, clock=clock_b)
    # suffix publication: the reference's whole-chain publication under the
    # hit node lets eviction free blocks still pinned by live sequences
    eng = BatchedKVEngine(cache, n_q_heads=HQ, free_private_blocks=True,
                          publish_mode=publish_mode)
    ref = OracleEngine(meta, free_private=True, suffix_publish=publish_mode == "suffix")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    shadow = {}
    next_id = [0]

    def prefill(ids, prompts, base):
        for sid, toks in zip(ids, prompts):
            eng.add(sid, toks)
            ref.add(sid, toks)
        q = [len(t) - eng.seqs[s].n_tokens for s, t in zip(ids, prompts)]
        p = eng.plan(ids, q, attend=False)
        ref.step(ids, q)
        k, v = _randn((sum(q), HK, D), g), _randn((sum(q), HK, D), g)
        eng.append(p, 0, k, v)
        o = 0
        for sid, n0, qi in zip(ids, p.n_past, q):
            pk, pv = base.get(sid, (k[:0], v[:0]))
            shadow[sid] = (torch.cat([pk[:n0], k[o:o + qi]]), torch.cat([pv[:n0], v[o:o + qi]]))
            o += qi
        eng.commit(p)
        ref.commit(ids, q)

    def new_ids(n):
        out = list(range(next_id[0], next_id[0] + n))
        next_id[0] += n
        return out

    # popular prefixes: written once, published, owned by the tree
    pref_tok = [[900000 + 10000 * j + i for i in range(1024)] for j in range(4)]
    wid = new_ids(4)
    prefill(wid, pref_tok, {})
    pref_kv = {j: shadow.pop(w) for j, w in enumerate(wid)}
    for w in wid:
        eng.finish(w)
        ref.finish(w)

    def prompts_for(ctxs):
        ps, base = [], {}
        for c in ctxs:
            c = max(int(c), 2)
            if rng.random() < 0.5:
                j = int(rng.integers(0, 4))
                extra = max(1, c - 1024)
                ps.append(pref_tok[j] + [int(x) for x in rng.integers(0, 50000, size=extra)])
                base[len(ps) - 1] = pref_kv[j]
            else:
                ps.append([int(x) for x in rng.integers(0, 50000, size=c)])
        return ps, base

    def admit(ctxs):
        ids = new_ids(len(ctxs))
        ps, b = prompts_for(ctxs)
        prefill(ids, ps, {ids[i]: kv for i, kv in b.items()})

    def check_meta():
        assert {k: (s.block_table, s.n_tokens) for k, s in eng.seqs.items()} == \
            {k: (s["table"], s["n"]) for k, s in ref.seqs.items()}
        assert list(cache._free) == list(meta._free)
        assert tree_sig(cache._root) == tree_sig(meta._root)

    admit([ctx_all[i] for i in share])
    check_meta()
    moved_total = 0
    for step in range(3):
        live = sorted(eng.seqs)
        pool_ids = live if publish_mode == "suffix" else \
            [sid for sid in live if eng.seqs[sid].radix_node is None]
        done = [pool_ids[i] for i in rng.choice(len(pool_ids), size=max(1, len(live) // 20),
                                                replace=False)]
        for sid in done:
            eng.finish(sid)
            ref.finish(sid)
            shadow.pop(sid)
        admit([next(new_ctx) for _ in done])
        k_ev = int(rng.integers(16, 256))
        live_blocks = {b for s in eng.seqs.values() for b in s.block_table}
        free_before = set(cache._free)
        assert cache.evict(k_ev) == meta.evict(k_ev)
        freed = set(cache._free) - free_before
        assert not freed & live_blocks, "eviction freed blocks of live sequences"
        moved = eng.compact()
        assert moved == len(ref.compact())
        moved_total += moved
        check_meta()
        # one decode step for every live sequence
        ids = sorted(eng.seqs)
        p = eng.plan(ids)
        ref.step(ids, [1] * len(ids))
        k, v = _randn((len(ids), HK, D), g), _randn((len(ids), HK, D), g)
        q = _randn((len(ids), HQ, D), g)
        eng.append(p, 0, k, v)
        out = eng.attend(p, 0, q).cpu().numpy()
        eng.commit(p)
        ref.commit(ids, [1] * len(ids))
        for i, sid in enumerate(ids):
            sk, sv = shadow[sid]
            shadow[sid] = (torch.cat([sk, k[i:i + 1]]), torch.cat([sv, v[i:i + 1]]))
        check_meta()
        assert np.isfinite(out).all()
        for i in sorted(set(int(x) for x in rng.choice(len(ids), size=6, replace=False))):
            sid = ids[i]
            s = eng.seqs[sid]
            kb, vb = pool_rows(cache, 0, s.block_table, 0, s.n_tokens)
            sk, sv = (t.float().cpu().numpy() for t in shadow[sid])
            assert np.array_equal(kb, sk) and np.array_equal(vb, sv), f"seq {sid} K/V"
            ref_rows = oracle_rows(q[i:i + 1].float().cpu().numpy(), sk, sv)
            assert_close_rows(out[i:i + 1], ref_rows, BF16_RTOL, f"seq {sid}")
    assert moved_total > 0


# ---------------------------------------------------------------------------
# engine: shared partial tail (copy-on-write), verify chain, rollback, re-verify
# ---------------------------------------------------------------------------
def test_engine_shared_tail_verify_rollback():
    from chenxing_b200 import RadixPagedKVCache
    from chenxing_b200.engine import BatchedKVEngine

    cache = RadixPagedKVCache(64, BS, 2, HK, D, dtype="bfloat16", host_io=False)
    eng = BatchedKVEngine(cache, n_q_heads=HQ, window=24)
    g = torch.Generator(device="cuda")
    g.manual_seed(8)
    rng = np.random.default_rng(8)
    donor = [int(x) for x in rng.integers(0, 1000, size=37)]
    eng.add(0, donor)
    p = eng.plan([0], [37], attend=False)
    kv0 = _randn((2, 2, 37, HK, D), g)
    for l in range(2):
        eng.append(p, l, kv0[0, l], kv0[1, l])
    eng.commit(p)
    assert eng.publish(0)                          # blocks 0-1 into the tree
    shared = list(eng.seqs[0].block_table)
    s1 = eng.add(1, donor + [5, 6, 7, 8], share_tail_from=0)
    assert s1.n_tokens == 37 and s1.block_table == shared[:3] and s1.aliased == {2}
    hist = {0: [kv0[:, :, :37]], 1: [kv0[:, :, :37]]}

    def step(q_lens):
        ids = [0, 1]
        p = eng.plan(ids, q_lens)
        rows = sum(q_lens)
        kv = _randn((2, 2, rows, HK, D), g)
        q = _randn((2, rows, HQ, D), g)
        outs = []
        for l in range(2):
            eng.append(p, l, kv[0, l], kv[1, l])
            outs.append(eng.attend(p, l, q[l]).cpu().numpy())
        o = 0
        for sid, n0, ql in zip(ids, p.n_past, q_lens):
            cur = torch.cat(hist[sid], dim=2)[:, :, :n0]
            hist[sid] = [cur, kv[:, :, o:o + ql]]
            full = torch.cat(hist[sid], dim=2)
            for l in range(2):
                kb, vb = pool_rows(cache, l, eng.seqs[sid].block_table, 0, n0 + ql)
                assert np.array_equal(kb, full[0, l].float().cpu().numpy())
                assert np.array_equal(vb, full[1, l].float().cpu().numpy())
                ref = oracle_rows(q[l, o:o + ql].float().cpu().numpy(),
                                  full[0, l].float().cpu().numpy(),
                                  full[1, l].float().cpu().numpy(), window=24)
                assert_close_rows(outs[l][o:o + ql], ref, BF16_RTOL, f"seq {sid} layer {l}")
            o += ql
        eng.commit(p)
        return p

    p = step([1, 4])
    # both wrote into the aliased block: the first writer got a private copy
    assert len(p.cow_host) == 1 and p.cow_host[0][0] == shared[2] and p.cow_host[0][2] == 5
    assert eng.seqs[0].block_table[2] != eng.seqs[1].block_table[2]
    assert eng.seqs[0].block_table[:2] == eng.seqs[1].block_table[:2] == shared[:2]
    eng.rollback(1, 38)                            # 3 of 4 verify rows rejected
    assert eng.seqs[1].n_tokens == 38
    step([2, 5])
    assert eng.seqs[1].n_tokens == 43


def test_engine_append_rope_then_verify_matches_oracle():
    """BatchedKVEngine.append_rope positions each token at its sequence's
    committed length + index (transformer.py:84-87 with positions =
    n_past + arange(T)); Q and K rotated, then verify attention."""
    from chenxing_b200 import RadixPagedKVCache, RopeTables
    from chenxing_b200.engine import BatchedKVEngine
    from oracle.rope import rotate

    cache = RadixPagedKVCache(64, BS, 1, HK, D, dtype="bfloat16", host_io=False)
    eng = BatchedKVEngine(cache, n_q_heads=HQ)
    rope = RopeTables(4096, D, 500000.0)
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    rng = np.random.default_rng(12)
    prompts = [[int(x) for x in rng.integers(0, 1000, size=n)] for n in (70, 33)]
    hist = {}
    for sid, pr in enumerate(prompts):
        eng.add(sid, pr)
    for step_q in ([70, 33], [5, 9]):
        p = eng.plan([0, 1], step_q)
        rows = sum(step_q)
        k, v = _randn((rows, HK, D), g, 1.0), _randn((rows, HK, D), g, 1.0)
        q = _randn((rows, HQ, D), g, 1.0)
        qr = eng.append_rope(p, 0, k, v, rope, q=q)
        out = eng.attend(p, 0, qr).cpu().numpy()
        cos, sin = rope.cos.cpu().numpy(), rope.sin.cpu().numpy()
        o = 0
        for sid, (n0, ql) in enumerate(zip(p.n_past, step_q)):
            pos = np.arange(n0, n0 + ql)
            kr = bf16_round(rotate(k[o:o + ql].float().cpu().numpy(), cos, sin, pos))
            hist[sid] = np.concatenate([hist.get(sid, np.zeros((0, HK, D), np.float32)), kr])
            vv = np.concatenate([hist.get(("v", sid), np.zeros((0, HK, D), np.float32)),
                                 v[o:o + ql].float().cpu().numpy()])
            hist[("v", sid)] = vv
            qref = bf16_round(rotate(q[o:o + ql].float().cpu().numpy(), cos, sin, pos))
            assert np.array_equal(qr[o:o + ql].float().cpu().numpy(), qref)
            ref = oracle_rows(qref, hist[sid], vv)
            assert_close_rows(out[o:o + ql], ref, BF16_RTOL, f"seq {sid}")
            o += ql
        eng.commit(p)
