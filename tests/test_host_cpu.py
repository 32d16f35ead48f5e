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


def test_partition_by_context_is_balanced_and_complete():
    from chenxing_b200.workloads import lognormal_ctx
    ctx = lognormal_ctx(1024, seed=3)
    groups = partition_by_context(ctx, 8)
    flat = sorted(i for g in groups for i in g)
    assert flat == list(range(1024))
    loads = [int(ctx[g].sum()) for g in groups]
    assert max(loads) - min(loads) <= int(ctx.max())
