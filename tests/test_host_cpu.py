"""CPU-only tests: library symbols, host-side metadata logic, sharding."""
import ctypes
import os
import re

import numpy as np
import pytest

from chenxing_b200 import _lib
from chenxing_b200.batch import slot_mapping
from chenxing_b200.radix_kv import OutOfKVCacheError, RadixIndex
from chenxing_b200.seqmeta import grow_table, rollback
from chenxing_b200.sharding import partition_by_context
from oracle.radix_kv import logical_clock
from replay import load_json, replay_radix

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "cxkv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cx_[a-z_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 10
    lib = _lib.load_library()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/cxkv.h but not exported"
        assert n in _lib.EXPORTS
    assert lib.cx_version().startswith(b"cxkv")


def test_kernel_selection_rules_read_host_fields_only():
    """cx_paged_kernel_kind decides from host fields alone, so the dispatch
    rules hold without a GPU: bf16 pools with 16-token blocks and head_dim 64 /
    128 take mma.sync below 64 packed rows (query tokens x GQA group) and
    tcgen05 from 64 rows; fp32 pools with 16-token blocks and head_dim 64 /
    128 take the fp32 FMA kernel up to 64 packed rows; fp16 pools, other
    block sizes or head dims, longer fp32 query tiles and pools not 16-byte
    aligned take the generic kernel.  The pool and table addresses are
    placeholders that nothing dereferences."""
    lib = _lib.load_library()

    def kind(*, dtype=_lib.CX_BF16, bs=16, d=128, hk=8, hq=32, q=1, verify=1,
             q_dtype=_lib.CX_BF16, base=0x100000):
        pool = _lib.CxPool(base, base + 0x4000000, 2, 1024, bs, hk, d, dtype, 0)
        b = _lib.CxAttnBatch(0x200000, 64, 0x300000, 0x400000 if verify else None, 4, q,
                             hq, float("nan"), 0, 0)
        return _lib.KERNEL_KINDS[lib.cx_paged_kernel_kind(ctypes.byref(pool), ctypes.byref(b),
                                                          q_dtype, verify)]

    assert kind(verify=0) == "mma"                      # decode: G = 4 rows
    assert kind(verify=0, q=50) == "mma"                # decode ignores max_q_len
    assert kind(q=15) == "mma" and kind(q=16) == "tcgen05"   # 60 / 64 packed rows
    assert kind(q=9) == kind(q=9, d=64) == "mma"        # 36 rows, both head dims
    assert kind(hq=8, hk=8, q=63) == "mma" and kind(hq=8, hk=8, q=64) == "tcgen05"
    assert kind(q=200, q_dtype=_lib.CX_F32) == "tcgen05"
    assert kind(q=200, q_dtype=_lib.CX_F16) == "generic"
    f32 = dict(dtype=_lib.CX_F32)
    assert kind(verify=0, **f32) == kind(verify=0, d=64, **f32) == "fma"
    assert kind(q=16, **f32) == "fma" and kind(q=17, **f32) == "generic"   # 64 / 68 rows
    assert kind(q=4, q_dtype=_lib.CX_F32, **f32) == "fma"
    assert kind(q=4, q_dtype=_lib.CX_F16, **f32) == "generic"
    for bad in (dict(dtype=_lib.CX_F16), dict(bs=32), dict(d=96), dict(d=256),
                dict(base=0x100008), dict(dtype=_lib.CX_F32, bs=8),
                dict(dtype=_lib.CX_F32, d=32), dict(dtype=_lib.CX_F32, base=0x100008)):
        assert kind(**bad) == "generic", bad
        assert kind(q=100, **bad) == "generic", bad


def test_struct_layouts_match_header():
    assert ctypes.sizeof(_lib.CxPool) == 2 * 8 + 5 * 8 + 2 * 4
    assert ctypes.sizeof(_lib.CxAttnBatch) == 8 * 7 + 4 + 4 + 8


def test_radix_index_replays_reference_bit_exact():
    fx = load_json("radix_ops.json")
    idx = RadixIndex(fx["n_blocks"], fx["block_size"], clock=logical_clock())
    bad = replay_radix(idx, fx, OutOfKVCacheError)
    assert not bad, "\n".join(bad)


def test_block_tables_slots_and_rollback_match_reference():
    fx = load_json("engine_meta.json")
    bs = fx["block_size"]
    idx = RadixIndex(fx["n_blocks"], bs, clock=logical_clock())
    tables = [[] for _ in range(fx["n_seqs"])]
    n_tok = [0] * fx["n_seqs"]
    for step in fx["trace"]:
        i, t = step["seq"], step["t"]
        grow_table(idx, tables[i], n_tok[i] + t)
        assert slot_mapping([tables[i]], [n_tok[i]], [t], bs).tolist() == step["slots"]
        n_tok[i] = rollback(n_tok[i] + t, n_tok[i] + t - step["rejected"])
        assert tables[i] == step["table"] and n_tok[i] == step["n_tokens"]
        assert list(idx._free) == step["free"]


# The reference's own tests/test_radix_kv.py, logical-layer cases, on RadixIndex.
def make_index(n_blocks=8, block_size=4):
    return RadixIndex(n_blocks, block_size)


def test_block_pool_bounds_and_free_accounting():
    c = make_index(n_blocks=4)
    ids = [c.alloc_block() for _ in range(4)]
    assert len(set(ids)) == 4 and c.free_blocks == 0
    with pytest.raises(OutOfKVCacheError):
        c.alloc_block()
    c._free_block(ids[0])
    assert c.free_blocks == 1


def test_prefix_match_zero_copy_share():
    c = make_index()
    toks = [1, 2, 3, 4, 5, 6, 7, 8]
    node = c.insert(toks, [c.alloc_block(), c.alloc_block()])
    hit = c.match_prefix(toks)
    assert hit.n_tokens == 8 and hit.block_ids == node.blocks
    hit2 = c.match_prefix(toks[:4] + [99, 99, 99, 99])
    assert hit2.n_tokens == 4 and hit2.block_ids == node.blocks[:1]


def test_partial_prefix_does_not_overmatch():
    c = make_index()
    c.insert([1, 2, 3, 4], [c.alloc_block()])
    assert c.match_prefix([1, 2, 9, 9]).n_tokens == 0


def test_lru_eviction_and_pinning():
    c = make_index(n_blocks=4)
    n1 = c.insert([1, 2, 3, 4], [c.alloc_block()])
    c.insert([9, 9, 9, 9], [c.alloc_block()])
    c.acquire(n1)
    assert c.evict(2) == 1
    assert c.match_prefix([1, 2, 3, 4]).n_tokens == 4
    c.release(n1)
    c.evict(2)
    assert c.match_prefix([1, 2, 3, 4]).n_tokens == 0 and c.free_blocks == 4


def test_refcount_underflow_and_alignment_errors():
    c = make_index()
    n = c.insert([1, 2, 3, 4], [c.alloc_block()])
    with pytest.raises(RuntimeError):
        c.release(n)
    with pytest.raises(ValueError):
        c.insert([1, 2, 3], [c.alloc_block()])


def test_ensure_free_raises_when_all_pinned():
    c = make_index(n_blocks=2)
    n = c.insert([1, 2, 3, 4, 5, 6, 7, 8], [c.alloc_block(), c.alloc_block()])
    c.acquire(n)
    with pytest.raises(OutOfKVCacheError):
        c.ensure_free(1)


def test_slot_mapping_rejects_short_table():
    with pytest.raises(ValueError):
        slot_mapping([[0]], [0], [3], 2)


def test_slot_mapping_matches_the_placement_rule():
    """slot = table[p // bs] * bs + p % bs for every written position
    (radix_kv.py:123-128), over ragged tables, empty write ranges and ranges
    that start mid-block."""
    rng = np.random.default_rng(4)
    for trial in range(200):
        bs = int(rng.choice([1, 2, 16]))
        B = int(rng.integers(0, 9))
        tables, starts, counts = [], [], []
        for _ in range(B):
            n = int(rng.integers(0, 12))
            tables.append(rng.integers(0, 1000, size=n).tolist())
            cap = n * bs
            s = int(rng.integers(0, cap + 1))
            c = int(rng.integers(0, cap - s + 1)) if trial % 5 else 0
            starts.append(s)
            counts.append(c)
        want = [t[p // bs] * bs + p % bs
                for t, s, c in zip(tables, starts, counts) for p in range(s, s + c)]
        got = slot_mapping(tables, starts, counts, bs)
        assert got.dtype == np.int64
        assert got.tolist() == want


def test_free_list_keeps_the_reference_fifo_rules():
    """The free list against the reference's dict-as-ordered-set: allocation
    takes the oldest id, freeing appends, re-freeing a free id keeps its
    place, deleting an arbitrary id (compaction) drops it; order, length and
    membership agree after every operation of a random script."""
    rng = np.random.default_rng(11)
    n = 64
    idx = RadixIndex(n, 16)
    model = dict.fromkeys(range(n))
    for _ in range(5000):
        op = int(rng.integers(0, 6))
        if op == 0 and model:
            b = next(iter(model))
            del model[b]
            assert idx.alloc_block() == b
        elif op == 1:
            b = int(rng.integers(0, n))
            model[b] = None
            idx._free_block(b)
        elif op == 2 and model:
            b = int(rng.choice(list(model)))
            del model[b]
            del idx._free[b]
        elif op == 3:                       # batch allocation: the same ids, same order
            k = int(rng.integers(0, 6))
            if k > len(model):
                with pytest.raises(OutOfKVCacheError):
                    idx.alloc_blocks(k)
            else:
                want = list(model)[:k]
                for b in want:
                    del model[b]
                assert idx.alloc_blocks(k) == want
        elif op == 4:                       # batch free, repeats and already-free ids included
            ids = [int(x) for x in rng.integers(0, n, size=int(rng.integers(0, 6)))]
            for b in ids:
                model[b] = None
            idx._free_blocks(ids)
        assert len(idx._free) == len(model) == idx.free_blocks
        b = int(rng.integers(0, n))
        assert (b in idx._free) == (b in model)
    assert list(idx._free) == list(model)
    assert idx._free.mask().tolist() == [int(b in model) for b in range(n)]


def test_admission_router_is_replicable_balanced_and_conserving():
    """Two copies of the router built from the same arguments make the same
    finish and placement decisions (so ranks agree without messages); live
    sets stay disjoint and complete; the KV-token spread across ranks stays
    far below what independent per-rank admissions give."""
    from chenxing_b200.sharding import AdmissionRouter
    from chenxing_b200.workloads import lognormal_ctx
    ctx = lognormal_ctx(256, seed=3)
    groups = partition_by_context(ctx, 4)
    a, b = (AdmissionRouter(ctx, groups, 0.05, seed=9) for _ in range(2))
    stream = iter(lognormal_ctx(20000, seed=4))
    rng = np.random.default_rng(0)
    indep = [int(ctx[g].sum()) for g in groups]        # each rank refills on its own
    indep_live = [list(ctx[g]) for g in groups]
    for _ in range(60):
        fa, fb = a.finish_step(), b.finish_step()
        assert fa == fb
        new = [int(next(stream)) for _ in range(sum(len(f) for f in fa))]
        pa, pb = a.admit(new), b.admit(new)
        assert pa == pb
        assert [c for _, _, c in pa] == new
        a.grow()
        b.grow()
        live = [set(a.live(r)) for r in range(4)]
        assert sum(len(x) for x in live) == 256 and len(set().union(*live)) == 256
        for r in range(4):
            assert a.load[r] == sum(a.ctx[i] for i in live[r])
        for r in range(4):                              # the unrouted comparison
            k = max(1, round(0.05 * len(indep_live[r])))
            for _ in range(k):
                indep_live[r].pop(int(rng.integers(0, len(indep_live[r]))))
            indep_live[r] += [int(x) for x in lognormal_ctx(k, seed=int(rng.integers(1 << 30)))]
            indep[r] = sum(indep_live[r])
    assert max(a.load) / np.mean(a.load) < 1.02
    assert max(a.load) / np.mean(a.load) < max(indep) / np.mean(indep)


def test_deal_by_context_equal_counts_balanced_sums():
    """A global batch dealt to ranks by length: every rank gets the same
    number of sequences, every index exactly once, and the token sums differ
    by at most one round's largest length gap (far less than independent
    per-rank draws differ)."""
    from chenxing_b200.sharding import deal_by_context
    rng = np.random.default_rng(1)
    for world in (1, 2, 4, 8):
        ctx = rng.integers(1024, 8193, size=64 * world)
        groups = deal_by_context(ctx, world)
        assert all(len(g) == 64 for g in groups)
        assert sorted(i for g in groups for i in g) == list(range(64 * world))
        assert all(g == sorted(g) for g in groups)
        sums = [int(ctx[g].sum()) for g in groups]
        assert max(sums) - min(sums) <= 8192 - 1024
        if world == 1:
            assert groups == [list(range(64))]
    with pytest.raises(ValueError):
        deal_by_context([1, 2, 3], 2)


def test_partition_by_context_is_balanced_and_complete():
    from chenxing_b200.workloads import lognormal_ctx
    ctx = lognormal_ctx(1024, seed=3)
    groups = partition_by_context(ctx, 8)
    flat = sorted(i for g in groups for i in g)
    assert flat == list(range(1024))
    loads = [int(ctx[g].sum()) for g in groups]
    assert max(loads) - min(loads) <= int(ctx.max())


def _churned_pair(seed):
    """The product index and the oracle driven through the same random churn:
    allocations into per-sequence tables, published prefixes, LRU evictions
    and frees, leaving holes all over the id range."""
    from oracle.radix_kv import OraclePagedKVCache
    rng = np.random.default_rng(seed)
    nb, bs = 300, 4
    idx = RadixIndex(nb, bs, clock=logical_clock())
    orc = OraclePagedKVCache(nb, bs, 1, 1, 1, with_pool=False, clock=logical_clock())
    tabs, otabs = [], []
    for step in range(40):
        n = int(rng.integers(1, 9))
        t, ot = [], []
        grow_table(idx, t, n * bs)
        from oracle.paged import ensure_capacity
        ensure_capacity(orc, ot, n * bs)
        assert t == ot
        kind = rng.integers(0, 3)
        if kind == 0 and n >= 2:              # publish whole blocks in the tree;
            toks = [int(step * 1000 + i) for i in range((n - 1) * bs)]
            idx.insert(toks, t[:n - 1])       # the tree owns them from now on
            orc.insert(toks, ot[:n - 1])
            t, ot = t[n - 1:], ot[n - 1:]
        if kind == 1 and tabs:                # a sequence finishes and frees
            j = int(rng.integers(0, len(tabs)))
            for b in tabs.pop(j):
                idx._free_block(b)
            for b in otabs.pop(j):
                orc._free_block(b)
        if rng.random() < 0.3:
            k = int(rng.integers(1, 6))
            assert idx.evict(k) == orc.evict(k)
        tabs.append(t)
        otabs.append(ot)
    return idx, orc, tabs, otabs


@pytest.mark.parametrize("max_moves", [None, 0, 1, 7])
def test_compaction_plan_matches_oracle(max_moves):
    from oracle.paged import compact
    from replay import tree_sig
    for seed in range(3):
        idx, orc, tabs, otabs = _churned_pair(seed)
        n_used = idx.n_blocks - idx.free_blocks
        src, dst = idx.plan_compaction(tabs, max_moves)
        moves = compact(orc, otabs, max_moves)
        assert list(zip(src, dst)) == moves
        assert tabs == otabs
        assert list(idx._free) == list(orc._free)
        assert tree_sig(idx._root) == tree_sig(orc._root)
        if max_moves is None:
            live = {b for t in tabs for b in t}
            assert all(b < n_used for b in live)
            assert all(b >= n_used for b in idx._free)
        # a second full pass after a full pass moves nothing
        if max_moves is None:
            assert idx.plan_compaction(tabs) == ([], [])


@pytest.mark.parametrize("free_private,mode", [(False, "reference"), (True, "reference"),
                                               (True, "suffix")])
def test_batched_engine_metadata_matches_oracle_replay(free_private, mode):
    """Continuous-batching churn through BatchedKVEngine's host half (bare
    RadixIndex, no device): admissions with shared-prefix hits, batched
    decode / verify steps, finishes that publish their prefix, LRU eviction
    under pressure and compaction; every table, length, the free list and the
    radix tree equal the oracle's per-sequence replay after every step."""
    from chenxing_b200.engine import BatchedKVEngine
    from engine_replay import OracleEngine
    from oracle.radix_kv import OraclePagedKVCache
    from replay import tree_sig
    rng = np.random.default_rng(5)
    nb, bs = 400, 4
    idx = RadixIndex(nb, bs, clock=logical_clock())
    orc = OraclePagedKVCache(nb, bs, 1, 1, 1, with_pool=False, clock=logical_clock())
    eng = BatchedKVEngine(idx, n_q_heads=1, free_private_blocks=free_private,
                          publish_mode=mode)
    ref = OracleEngine(orc, free_private, suffix_publish=mode == "suffix")
    prefixes = [[7000 + 100 * p + i for i in range(3 * bs)] for p in range(3)]
    next_id = 0

    def admit():
        nonlocal next_id
        n = int(rng.integers(1, 30))
        toks = (prefixes[int(rng.integers(0, 3))] if rng.random() < 0.5 else []) + \
            [int(x) for x in rng.integers(0, 500, size=n)]
        eng.add(next_id, toks)
        ref.add(next_id, toks)
        q = len(toks) - eng.seqs[next_id].n_tokens
        try:
            p = eng.plan_host([next_id], [q])
        except OutOfKVCacheError:
            with pytest.raises(Exception):
                ref.step([next_id], [q])
            return
        ref.step([next_id], [q])
        eng.commit(p)
        ref.commit([next_id], [q])
        next_id += 1

    def check():
        assert {k: (s.block_table, s.n_tokens) for k, s in eng.seqs.items()} == \
            {k: (s["table"], s["n"]) for k, s in ref.seqs.items()}
        assert list(idx._free) == list(orc._free)
        assert tree_sig(idx._root) == tree_sig(orc._root)
        # the incremental block counts equal a full walk of the tree / tables
        from collections import Counter
        walk, stack = Counter(), [idx._root]
        while stack:
            n = stack.pop()
            walk.update(n.blocks)
            stack.extend(n.children.values())
        assert walk == idx._owned
        assert Counter(b for s in eng.seqs.values() for b in s.block_table) == eng._held

    for _ in range(12):
        admit()
    check()
    for step in range(25):
        ids = sorted(eng.seqs)
        q = [int(rng.integers(1, 6)) if step % 4 == 3 else 1 for _ in ids]
        try:
            p = eng.plan_host(ids, q)
        except OutOfKVCacheError:
            with pytest.raises(Exception):
                ref.step(ids, q)
            break
        ref.step(ids, q)
        eng.commit(p)
        ref.commit(ids, q)
        check()
        for sid in ids:
            if rng.random() < 0.15:
                for t in range(int(rng.integers(1, 4))):
                    eng.extend_tokens(sid, [int(rng.integers(0, 500))])
                    ref.seqs[sid]["tokens"].append(eng.seqs[sid].tokens[-1])
        for sid in list(eng.seqs):
            if rng.random() < 0.1:
                eng.finish(sid)
                ref.finish(sid)
        for _ in range(int(rng.integers(0, 4))):
            admit()
        if step % 5 == 4:
            k = int(rng.integers(1, 20))
            assert idx.evict(k) == orc.evict(k)
            assert eng.compact() == len(ref.compact())
        check()


@pytest.mark.parametrize("mode", ["reference", "suffix"])
def test_reference_publish_lets_eviction_free_pinned_blocks(mode):
    """The reference publishes a finished sequence's whole chain under its hit
    node (engine.py:201 -> radix_kv.py:187); evicting that duplicate node
    frees the hit path's blocks while another sequence still pins them.
    ``publish_mode="suffix"`` publishes only the part past the hit."""
    from chenxing_b200.engine import BatchedKVEngine
    idx = RadixIndex(32, 4, clock=logical_clock())
    eng = BatchedKVEngine(idx, n_q_heads=1, publish_mode=mode)
    prefix = list(range(100, 108))                       # two whole blocks
    t = []
    grow_table(idx, t, 8)
    idx.insert(prefix, t)
    eng.add(1, prefix + [1, 2, 3, 4, 5])
    eng.add(2, prefix + [9, 9, 9, 9, 9])
    for sid in (1, 2):
        eng.commit(eng.plan_host([sid], [5]))
    pinned = eng.seqs[1].block_table[:2]
    eng.finish(2)
    idx.evict(1)
    freed = [b for b in pinned if b in idx._free]
    assert bool(freed) == (mode == "reference")



def test_cow_slots_inside_the_copied_rows_are_rejected():
    """An append's copy-on-write copies and its token stores run in one
    launch, so no token may land inside a destination block's copied rows."""
    from chenxing_b200.radix_kv import _check_cow_slots
    cow = (np.array([3, 5]), np.array([4, 6]), np.array([7, 2]))
    _check_cow_slots(np.array([4 * 16 + 7, 6 * 16 + 2, 9 * 16, -1]), cow, 16)
    with pytest.raises(ValueError):
        _check_cow_slots(np.array([4 * 16 + 6]), cow, 16)
    with pytest.raises(ValueError):
        _check_cow_slots([6 * 16 + 1, 4 * 16 + 8], cow, 16)
