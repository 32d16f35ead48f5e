"""Block-pool + radix-tree oracle (NumPy) — TEST INFRASTRUCTURE ONLY.

Restates ``chenxing/engine/radix_kv.py`` (class ``RadixPagedKVCache``):

* pool allocation / zero fill and FIFO free list ........ ``:77-93``
* ``alloc_block`` / ``_free_block`` / ``free_blocks`` ..... ``:99-111``
* ``write_layer`` per-token scatter ........................ ``:113-128``
* ``read_layer`` full-block gather + tail ................. ``:130-144``
* ``match_prefix`` / ``insert`` / ``acquire`` / ``release`` ``:150-219``
* ``evict`` / ``ensure_free`` / ``_lru_leaf`` ............. ``:221-252``
* ``stats`` ................................................ ``:261-273``

The LRU timestamp source is injectable (``clock``) so both this oracle and the
product can run on the same logical clock; the reference uses
``time.monotonic`` (``:67,255``).  Reference quirks kept on purpose: an
already-free id handed back keeps its place in the FIFO (dict keys are
unique, ``:111``), and ``_lru_leaf`` may choose an interior node (``:243-252``).
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass

import numpy as np

__all__ = ["OracleOutOfKV", "OracleNode", "OracleHit", "OraclePagedKVCache",
           "logical_clock"]


class OracleOutOfKV(RuntimeError):
    """Pool exhausted (reference ``OutOfKVCacheError``, radix_kv.py:45)."""


def logical_clock(start: int = 0):
    """Deterministic strictly increasing clock for LRU parity runs."""
    counter = itertools.count(start)
    return lambda: float(next(counter))


class OracleNode:
    __slots__ = ("tokens", "blocks", "children", "parent", "refcnt", "last_access")

    def __init__(self, tokens, blocks, parent, now):
        self.tokens = tokens
        self.blocks = blocks
        self.children = {}
        self.parent = parent
        self.refcnt = 0
        self.last_access = now


@dataclass
class OracleHit:
    node: OracleNode
    block_ids: list
    n_tokens: int


class OraclePagedKVCache:
    def __init__(self, n_blocks, block_size, n_layers, n_kv_heads, head_dim,
                 dtype=np.float32, *, clock=None, with_pool=True):
        if block_size <= 0 or n_blocks <= 0 or n_layers <= 0:
            raise ValueError("n_blocks, block_size, n_layers must be positive")
        self.block_size, self.n_blocks, self.n_layers = block_size, n_blocks, n_layers
        self.n_kv_heads, self.head_dim, self.dtype = n_kv_heads, head_dim, dtype
        self._now = clock or logical_clock()
        if with_pool:
            shape = (n_layers, n_blocks, block_size, n_kv_heads, head_dim)
            self.k_pool = np.zeros(shape, dtype=dtype)
            self.v_pool = np.zeros(shape, dtype=dtype)
        self._free = dict.fromkeys(range(n_blocks))
        self._root = OracleNode([], [], None, self._now())
        self._hits = 0
        self._lookups = 0

    # ---------------- physical layer ---------------- #
    @property
    def free_blocks(self):
        return len(self._free)

    def free_list(self):
        return list(self._free)

    def alloc_block(self):
        if not self._free:
            raise OracleOutOfKV(f"KV cache exhausted ({self.n_blocks} blocks)")
        bid = next(iter(self._free))
        del self._free[bid]
        return bid

    def _free_block(self, bid):
        self._free[bid] = None

    def write_layer(self, block_table, slot_start, layer, k, v):
        n = k.shape[0]
        bs = self.block_size
        if len(block_table) * bs < slot_start + n:
            raise ValueError("block_table too short for requested write range")
        for t in range(n):
            p = slot_start + t
            self.k_pool[layer, block_table[p // bs], p % bs] = k[t]
            self.v_pool[layer, block_table[p // bs], p % bs] = v[t]

    def read_layer(self, block_table, n_tokens, layer):
        h, d = self.n_kv_heads, self.head_dim
        if n_tokens == 0 or not block_table:
            e = np.zeros((0, h, d), dtype=self.dtype)
            return e, e
        n = min(n_tokens, len(block_table) * self.block_size)
        nb = -(-n // self.block_size)
        ks = self.k_pool[layer, list(block_table[:nb])].reshape(-1, h, d)[:n]
        vs = self.v_pool[layer, list(block_table[:nb])].reshape(-1, h, d)[:n]
        return ks.copy(), vs.copy()

    # ---------------- logical layer ---------------- #
    def _touch(self, node):
        node.last_access = self._now()

    def match_prefix(self, token_ids):
        self._lookups += 1
        bs = self.block_size
        node, blocks, i = self._root, [], 0
        while i < len(token_ids):
            child = node.children.get(token_ids[i])
            if child is None:
                break
            seg = child.tokens
            lim = min(len(seg), len(token_ids) - i)
            n = 0
            while n < lim and token_ids[i + n] == seg[n]:
                n += 1
            full = n == len(seg)
            take = (len(seg) if full else n) // bs
            if take == 0:
                break
            blocks += child.blocks[:take]
            i += take * bs
            node = child
            if not full:
                break
        if i > 0:
            self._hits += 1
            self._touch(node)
        return OracleHit(node, blocks, i)

    def insert(self, token_ids, block_ids, parent=None):
        bs = self.block_size
        if len(token_ids) != len(block_ids) * bs:
            raise ValueError("insert requires block-aligned tokens/blocks")
        if parent is None:
            hit = self.match_prefix(token_ids)
            parent = hit.node
            token_ids = token_ids[hit.n_tokens:]
            block_ids = block_ids[hit.n_tokens // bs:]
        if not token_ids:
            self._touch(parent)
            return parent
        if not parent.children and parent.refcnt == 0 and parent is not self._root:
            parent.tokens.extend(token_ids)
            parent.blocks.extend(block_ids)
            self._touch(parent)
            return parent
        node = OracleNode(list(token_ids), list(block_ids), parent, self._now())
        parent.children[token_ids[0]] = node
        return node

    def acquire(self, node):
        while node is not None and node is not self._root:
            node.refcnt += 1
            self._touch(node)
            node = node.parent

    def release(self, node):
        while node is not None and node is not self._root:
            if node.refcnt <= 0:
                raise RuntimeError("refcount underflow")
            node.refcnt -= 1
            node = node.parent

    def _lru_leaf(self):
        best, stack = None, [self._root]
        while stack:
            n = stack.pop()
            for c in n.children.values():
                stack.append(c)
                if c.refcnt == 0 and (best is None or c.last_access < best.last_access):
                    best = c
        return best

    def evict(self, n_blocks_needed=1):
        freed = 0
        while freed < n_blocks_needed:
            victim = self._lru_leaf()
            if victim is None:
                return freed
            freed += len(victim.blocks)
            for b in victim.blocks:
                self._free_block(b)
            del victim.parent.children[victim.tokens[0]]
        return freed

    def ensure_free(self, n_needed):
        while self.free_blocks < n_needed:
            if self.evict(n_needed - self.free_blocks) == 0:
                raise OracleOutOfKV("no evictable blocks; all pinned")

    def stats(self):
        total, stack = 0, [self._root]
        while stack:
            n = stack.pop()
            total += len(n.children)
            stack.extend(n.children.values())
        return {"n_blocks": self.n_blocks, "free_blocks": self.free_blocks,
                "cached_blocks": self.n_blocks - self.free_blocks,
                "radix_nodes": total,
                "prefix_hit_rate": self._hits / max(self._lookups, 1)}

    def tree_signature(self):
        """Deterministic nested description of the tree (for parity checks)."""
        def walk(n):
            return [list(n.tokens), list(n.blocks), n.refcnt,
                    [[k, walk(c)] for k, c in n.children.items()]]
        return walk(self._root)
