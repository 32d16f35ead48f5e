"""RadixPagedKVCache with its physical block pool in HBM.

Drop-in for the reference class ``chenxing.engine.radix_kv.RadixPagedKVCache``
(``chenxing/engine/radix_kv.py:77-273``): same constructor, attributes, methods
and errors.  The logical layer (radix prefix tree, refcounts, LRU eviction,
FIFO free list) stays on the host in Python with the reference semantics,
bit-exact; the K/V pools are CUDA tensors and every data movement is a
libcxkv kernel:

* ``write_layer``  -> ``cx_kv_append``  (slot-mapped scatter, radix_kv.py:113-128)
* ``append_rope``  -> ``cx_kv_append_rope`` (apply_rope on Q and K fused into the
  scatter, transformer.py:84-87)
* ``read_layer``   -> ``cx_kv_gather``  (radix_kv.py:130-144)
* ``copy_blocks`` / ``cow_tail`` / ``compact`` -> ``cx_block_copy`` (no reference
  counterpart)
* ``append_batch`` / ``decode_batch`` / ``verify_batch`` — batched forms over
  many sequences (see ``chenxing_b200.batch``).

Physical layout: ``[n_layers][n_blocks][n_kv_heads][block_size][head_dim]``
per pool, so one (block, head) is one contiguous tile.  ``k_pool`` / ``v_pool``
expose the reference's axis order ``(n_layers, n_blocks, block_size,
n_kv_heads, head_dim)`` as a strided view of that storage.
"""
from __future__ import annotations

import time
from collections import Counter, deque
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._arrays import to_device, to_numpy, torch_dtype, upload

__all__ = ["RadixPagedKVCache", "RadixIndex", "PrefixHit", "OutOfKVCacheError"]


class OutOfKVCacheError(RuntimeError):
    """The physical block pool is exhausted (radix_kv.py:45)."""


class _FreeList:
    """FIFO free list of block ids with the reference's rules
    (radix_kv.py:90,107,111): allocation takes the oldest free id, freeing
    appends, and freeing an id that is already free keeps its place.

    A deque of (id, ticket) entries plus each free id's current ticket:
    removing an arbitrary id (compaction) only voids its ticket, and stale
    entries are dropped when they reach the front, so every operation is O(1)
    amortised.  (A dict used as an ordered set made taking the first id cost
    O(ids deleted since the dict last resized): ~4 us per allocation at a few
    thousand allocations a step.)  ``mask()`` is a uint8 view, 1 = free.
    Iteration, ``keys()``, ``in``, ``len`` and ``del`` behave as they did on
    that dict."""
    __slots__ = ("_q", "_ticket", "_flag", "_n", "_next")

    def __init__(self, n: int) -> None:
        self._q = deque(zip(range(n), range(n)))
        self._ticket = list(range(n))
        self._flag = bytearray(b"\x01") * n
        self._n = n
        self._next = n

    def __len__(self) -> int:
        return self._n

    def __contains__(self, bid) -> bool:
        return 0 <= bid < len(self._flag) and self._flag[bid] == 1

    def __iter__(self):
        flag, ticket = self._flag, self._ticket
        return (b for b, t in self._q if flag[b] and ticket[b] == t)

    def keys(self):
        return iter(self)

    def pop_first(self) -> int:
        q, flag, ticket = self._q, self._flag, self._ticket
        while True:
            b, t = q.popleft()
            if flag[b] and ticket[b] == t:
                flag[b] = 0
                self._n -= 1
                return b

    def pop_many(self, n: int) -> list:
        """The ``n`` oldest free ids, in order (the caller checked ``len``)."""
        q, flag, ticket = self._q, self._flag, self._ticket
        out = []
        while len(out) < n:
            b, t = q.popleft()
            if flag[b] and ticket[b] == t:
                flag[b] = 0
                out.append(b)
        self._n -= n
        return out

    def add(self, bid: int) -> None:
        self.add_many((bid,))

    def add_many(self, ids) -> None:
        """Free ``ids`` in order: each goes to the back unless already free."""
        flag, ticket, append = self._flag, self._ticket, self._q.append
        nxt = self._next
        for bid in ids:
            if flag[bid]:
                continue
            flag[bid] = 1
            ticket[bid] = nxt
            append((bid, nxt))
            nxt += 1
        self._n += nxt - self._next
        self._next = nxt
        if len(self._q) > 2 * len(flag) + 1024:           # drop stale entries
            self._q = deque((b, t) for b, t in self._q if flag[b] and ticket[b] == t)

    def __delitem__(self, bid: int) -> None:
        if bid not in self:
            raise KeyError(bid)
        self._flag[bid] = 0
        self._n -= 1

    def mask(self) -> np.ndarray:
        return np.frombuffer(self._flag, dtype=np.uint8)


class _RadixNode:
    """A radix-tree edge: a block-aligned token run and its physical blocks
    (radix_kv.py:57-71)."""
    __slots__ = ("tokens", "blocks", "children", "parent", "refcnt", "last_access")

    def __init__(self, tokens: list, blocks: list, parent, now: float) -> None:
        self.tokens = tokens
        self.blocks = blocks
        self.children: dict = {}
        self.parent = parent
        self.refcnt = 0
        self.last_access = now

    @property
    def is_leaf(self) -> bool:
        return not self.children


@dataclass
class PrefixHit:
    """Longest cached prefix (radix_kv.py:49-54)."""
    node: _RadixNode
    block_ids: list
    n_tokens: int


class RadixIndex:
    """Host-side metadata of the cache: FIFO free list + radix prefix tree.

    Pure Python with the reference semantics (radix_kv.py:90-111,150-273);
    ``RadixPagedKVCache`` adds the HBM block pool on top.  ``clock`` replaces
    ``time.monotonic`` as the LRU timestamp source (for deterministic runs).
    """

    def __init__(self, n_blocks: int, block_size: int, clock=None) -> None:
        if block_size <= 0 or n_blocks <= 0:
            raise ValueError("n_blocks, block_size, n_layers must be positive")
        self.block_size = int(block_size)
        self.n_blocks = int(n_blocks)
        self._clock = clock or time.monotonic
        # FIFO free list; re-freeing a free id keeps its position
        # (radix_kv.py:90,107,111).
        self._free = _FreeList(self.n_blocks)
        self._root = _RadixNode([], [], None, self._clock())
        self._hits = 0
        self._lookups = 0
        # block id -> references from nodes reachable from the root, kept by
        # insert / evict / plan_compaction (what a walk of the tree would give)
        self._owned: Counter = Counter()

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def alloc_block(self) -> int:
        if not self._free:
            raise OutOfKVCacheError(
                f"KV cache exhausted ({self.n_blocks} blocks); scheduler must preempt")
        return self._free.pop_first()

    def _free_block(self, bid: int) -> None:
        self._free.add(bid)

    def alloc_blocks(self, n: int) -> list:
        """``n`` ``alloc_block`` calls in one: the same ids in the same order."""
        if n > len(self._free):
            raise OutOfKVCacheError(
                f"KV cache exhausted ({self.n_blocks} blocks); scheduler must preempt")
        return self._free.pop_many(n) if n > 0 else []

    def _free_blocks(self, ids) -> None:
        """``_free_block`` for each id, in order."""
        self._free.add_many(ids)

    def _touch(self, node: _RadixNode) -> None:
        node.last_access = self._clock()

    def match_prefix(self, token_ids: list) -> PrefixHit:
        """Longest block-aligned cached prefix, zero-copy (radix_kv.py:150-180)."""
        self._lookups += 1
        bs = self.block_size
        node, blocks, i = self._root, [], 0
        n_total = len(token_ids)
        while i < n_total:
            child = node.children.get(token_ids[i])
            if child is None:
                break
            seg = child.tokens
            limit = min(len(seg), n_total - i)
            n = 0
            while n < limit and token_ids[i + n] == seg[n]:
                n += 1
            whole = n == len(seg)
            n_take = (len(seg) if whole else n) // bs
            if n_take == 0:
                break
            blocks.extend(child.blocks[:n_take])
            i += n_take * bs
            node = child
            if not whole:
                break
        if i > 0:
            self._hits += 1
            self._touch(node)
        return PrefixHit(node, blocks, i)

    def insert(self, token_ids: list, block_ids: list, parent: _RadixNode | None = None):
        """Insert a block-aligned chain, sharing what exists (radix_kv.py:182-203)."""
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
        if parent.is_leaf and parent.refcnt == 0 and parent is not self._root:
            parent.tokens.extend(token_ids)
            parent.blocks.extend(block_ids)
            self._owned.update(block_ids)
            self._touch(parent)
            return parent
        child = _RadixNode(list(token_ids), list(block_ids), parent, self._clock())
        old = parent.children.get(token_ids[0])
        parent.children[token_ids[0]] = child
        if old is not None:                   # a replaced sibling drops out of the tree
            self._disown(old)
        self._owned.update(block_ids)
        return child

    def _disown(self, node: _RadixNode) -> None:
        """``node`` and its subtree left the tree: drop their block references."""
        stack = [node]
        while stack:
            n = stack.pop()
            self._owned.subtract(n.blocks)
            for b in n.blocks:
                if self._owned[b] <= 0:
                    del self._owned[b]
            stack.extend(n.children.values())

    def tree_holds(self, block_id: int) -> bool:
        """Whether a node reachable from the root lists ``block_id``."""
        return block_id in self._owned

    def acquire(self, node: _RadixNode) -> None:
        """Pin ``node`` and its ancestors (radix_kv.py:205-211)."""
        n = node
        while n is not None and n is not self._root:
            n.refcnt += 1
            self._touch(n)
            n = n.parent

    def release(self, node: _RadixNode) -> None:
        """Unpin; raises RuntimeError on underflow (radix_kv.py:213-219)."""
        n = node
        while n is not None and n is not self._root:
            if n.refcnt <= 0:
                raise RuntimeError("refcount underflow")
            n.refcnt -= 1
            n = n.parent

    def evict(self, n_blocks_needed: int = 1) -> int:
        """LRU-evict refcnt-0 nodes until enough blocks are free (radix_kv.py:221-235)."""
        freed = 0
        while freed < n_blocks_needed:
            victim = self._lru_leaf()
            if victim is None:
                return freed
            freed += len(victim.blocks)
            self._free_blocks(victim.blocks)
            del victim.parent.children[victim.tokens[0]]
            self._disown(victim)
        return freed

    def ensure_free(self, n_needed: int) -> None:
        """Evict until ``n_needed`` blocks are free (radix_kv.py:237-241)."""
        while self.free_blocks < n_needed:
            if self.evict(n_needed - self.free_blocks) == 0:
                raise OutOfKVCacheError("no evictable blocks; all pinned")

    def _lru_leaf(self) -> _RadixNode | None:
        """Least-recently-used refcnt-0 node over the whole tree, DFS order on
        ties; may be an interior node (radix_kv.py:243-252)."""
        best = None
        stack = [self._root]
        while stack:
            n = stack.pop()
            for c in n.children.values():
                stack.append(c)
                if c.refcnt == 0 and (best is None or c.last_access < best.last_access):
                    best = c
        return best

    def plan_compaction(self, tables=(), max_moves: int | None = None) -> tuple[list, list]:
        """Relabel in-use blocks so they pack into the lowest ids.

        No reference counterpart (the reference never moves data).  In use =
        not on the free list, so blocks the reference leaks (finished
        sequences' private blocks) are moved like any other.  With
        ``n_used = n_blocks - free_blocks``, every in-use id >= n_used is
        paired, highest first, with a free id < n_used, lowest first; at most
        ``max_moves`` pairs.  Radix-node block lists and every table in
        ``tables`` (lists of ids, edited in place) are rewritten; the free
        list keeps its surviving ids in FIFO order and then takes the vacated
        ids in ascending order.  Returns (src, dst) for the data copy, which
        the caller must issue before any further write to a dst block.
        Every live block table must be passed, or it keeps stale ids.
        """
        n_used = self.n_blocks - len(self._free)
        free = self._free.mask()
        n = int(max_moves) if max_moves is not None else self.n_blocks
        # free ids below n_used, lowest first; in-use ids from n_used, highest first
        holes = np.flatnonzero(free[:n_used])[:max(0, n)].tolist()
        high = (np.flatnonzero(free[n_used:] == 0)[::-1][:len(holes)] + n_used).tolist()
        n = min(len(holes), len(high))
        src, dst = high[:n], holes[:n]
        if not n:
            return [], []
        remap = dict(zip(src, dst))
        lo = min(src)                       # lists without an id >= lo keep their ids
        stack = [self._root]
        while stack:
            node = stack.pop()
            if node.blocks and max(node.blocks) >= lo:
                node.blocks[:] = [remap.get(b, b) for b in node.blocks]
            stack.extend(node.children.values())
        for t in tables:
            if t and max(t) >= lo:
                t[:] = [remap.get(b, b) for b in t]
        for a, b in remap.items():
            if a in self._owned:
                self._owned[b] += self._owned.pop(a)
        for d in dst:
            del self._free[d]
        self._free.add_many(sorted(src))
        return src, dst

    def stats(self) -> dict:
        total, stack = 0, [self._root]
        while stack:
            n = stack.pop()
            total += len(n.children)
            stack.extend(n.children.values())
        return {"n_blocks": self.n_blocks, "free_blocks": self.free_blocks,
                "cached_blocks": self.n_blocks - self.free_blocks, "radix_nodes": total,
                "prefix_hit_rate": self._hits / max(self._lookups, 1)}


def _check_cow_slots(slots, cow, block_size: int) -> None:
    """Raise ValueError if a slot lands inside the copied prefix of a
    copy-on-write destination block (the copy and the stores of one append
    launch run concurrently).  Device tensors are not inspected: reading them
    would synchronise the stream."""
    if any(isinstance(x, torch.Tensor) and x.is_cuda for x in (slots, *cow)):
        return
    s = np.asarray(slots.numpy() if isinstance(slots, torch.Tensor) else slots,
                   dtype=np.int64).reshape(-1)
    _, dst, nv = (np.asarray(c.numpy() if isinstance(c, torch.Tensor) else c,
                             dtype=np.int64).reshape(-1) for c in cow)
    live = s[s >= 0]
    blk, off = live // block_size, live % block_size
    for d, n in zip(dst, nv):
        if np.any((blk == d) & (off < n)):
            raise ValueError(f"copy-on-write: a slot of block {int(d)} falls inside its "
                             f"{int(n)} copied rows")


class RadixPagedKVCache(RadixIndex):
    """Physical block pool (all layers, in HBM) + logical radix prefix tree."""

    def __init__(self, n_blocks: int, block_size: int, n_layers: int, n_kv_heads: int,
                 head_dim: int, dtype=np.float32, *, device=None, host_io: bool = True,
                 clock=None) -> None:
        if block_size <= 0 or n_blocks <= 0 or n_layers <= 0:
            raise ValueError("n_blocks, block_size, n_layers must be positive")
        if n_kv_heads <= 0 or head_dim <= 0:
            raise ValueError("n_kv_heads and head_dim must be positive")
        self.device = _lib.require_cuda(device)
        _lib.lib()
        super().__init__(n_blocks, block_size, clock)
        self.n_layers = int(n_layers)
        self.n_kv_heads = int(n_kv_heads)
        self.head_dim = int(head_dim)
        self.dtype = dtype
        self.torch_dtype = torch_dtype(dtype)
        self.host_io = host_io
        shape = (self.n_layers, self.n_blocks, self.n_kv_heads, self.block_size, self.head_dim)
        with torch.cuda.device(self.device):
            self._k = torch.zeros(shape, dtype=self.torch_dtype, device=self.device)
            self._v = torch.zeros(shape, dtype=self.torch_dtype, device=self.device)
        self._pool = _lib.CxPool(self._k.data_ptr(), self._v.data_ptr(), self.n_layers,
                                 self.n_blocks, self.block_size, self.n_kv_heads,
                                 self.head_dim, _lib.cx_dtype(self.torch_dtype), 0)

    # ------------------------------------------------------------------ #
    # pool views
    # ------------------------------------------------------------------ #
    @property
    def k_pool(self) -> torch.Tensor:
        """K pool in the reference's axis order (L, NB, bs, H, D), a view."""
        return self._k.permute(0, 1, 3, 2, 4)

    @property
    def v_pool(self) -> torch.Tensor:
        return self._v.permute(0, 1, 3, 2, 4)

    @property
    def pool_bytes(self) -> int:
        return 2 * self._k.numel() * self._k.element_size()

    def cx_pool(self) -> _lib.CxPool:
        return self._pool

    # ------------------------------------------------------------------ #
    # physical layer (radix_kv.py:113-144)
    # ------------------------------------------------------------------ #
    def _check_ids(self, ids) -> None:
        for b in ids:
            if not 0 <= int(b) < self.n_blocks:
                raise IndexError(f"block id {b} outside [0, {self.n_blocks})")

    def write_layer(self, block_table: list, slot_start: int, layer: int, k, v) -> None:
        """Store K/V rows for positions [slot_start, slot_start + T) of one layer.

        k, v: (T, n_kv_heads, head_dim), NumPy or torch.  Position p lands in
        block ``block_table[p // block_size]`` at slot ``p % block_size``
        (radix_kv.py:113-128); values are rounded to the pool dtype (RNE).
        """
        t_total = int(k.shape[0])
        if len(block_table) * self.block_size < slot_start + t_total:
            raise ValueError("block_table too short for requested write range")
        if not 0 <= layer < self.n_layers:
            raise IndexError(f"layer {layer} outside [0, {self.n_layers})")
        if t_total == 0:
            return
        pos = np.arange(slot_start, slot_start + t_total, dtype=np.int64)
        bt = np.asarray(block_table, dtype=np.int64)
        used = bt[pos // self.block_size]
        self._check_ids(np.unique(used))
        slots = used * self.block_size + pos % self.block_size
        kt = to_device(k, self.device)
        vt = to_device(v, self.device)
        shape = (t_total, self.n_kv_heads, self.head_dim)
        if tuple(kt.shape) != shape or tuple(vt.shape) != shape:
            raise ValueError(f"k/v must have shape {shape}, got {tuple(kt.shape)} / {tuple(vt.shape)}")
        st = upload(slots, self.device)
        self.append_slots(layer, kt, vt, st)

    def append_slots(self, layer: int, k: torch.Tensor, v: torch.Tensor,
                     slot_mapping: torch.Tensor, cow=None) -> None:
        """Batched append: row t of k/v (device, [T, H, D]) goes to
        ``slot_mapping[t]`` (int64, device; negative = skip).  ``cow`` is an
        optional (src, dst, n_valid) triple of int32 device tensors: copy the
        first n_valid slots of block src into block dst for this layer first.
        """
        if cow is not None:
            cs, cd, cn = cow
            n_cow = int(cs.numel())
        else:
            cs = cd = cn = None
            n_cow = 0
        if slot_mapping.dtype != torch.int64:
            slot_mapping = slot_mapping.to(torch.int64)
        _lib.check(_lib.lib().cx_kv_append(
            self._pool, int(layer), k.data_ptr(), v.data_ptr(), _lib.cx_dtype(k.dtype),
            slot_mapping.data_ptr(), int(slot_mapping.numel()), _lib.ptr(cs), _lib.ptr(cd),
            _lib.ptr(cn), n_cow, _lib.stream_ptr(self.device)), "cx_kv_append")

    def read_layer(self, block_table: list, n_tokens: int, layer: int):
        """K/V of the first ``n_tokens`` positions, each (n, H, D) (radix_kv.py:130-144)."""
        h, d = self.n_kv_heads, self.head_dim
        if n_tokens == 0 or not block_table:
            e = torch.zeros((0, h, d), dtype=self.torch_dtype, device=self.device)
            return (to_numpy(e), to_numpy(e)) if self.host_io else (e, e.clone())
        n = min(int(n_tokens), len(block_table) * self.block_size)
        if not 0 <= layer < self.n_layers:
            raise IndexError(f"layer {layer} outside [0, {self.n_layers})")
        nb = -(-n // self.block_size)
        self._check_ids(block_table[:nb])
        table = torch.tensor(list(block_table[:nb]), dtype=torch.int32, device=self.device)
        ko = torch.empty((n, h, d), dtype=self.torch_dtype, device=self.device)
        vo = torch.empty_like(ko)
        _lib.check(_lib.lib().cx_kv_gather(self._pool, int(layer), table.data_ptr(), n,
                                           ko.data_ptr(), vo.data_ptr(),
                                           _lib.stream_ptr(self.device)), "cx_kv_gather")
        if self.host_io:
            return to_numpy(ko), to_numpy(vo)
        return ko, vo

    def copy_blocks(self, src: list, dst: list, n_slots: int | None = None,
                    events=None) -> None:
        """Copy slots [0, n_slots) of block src[i] into block dst[i], every layer,
        K and V (eviction compaction / prefix forking).  ``events``: an optional
        pair of CUDA events recorded right before and after the copy launch."""
        if len(src) != len(dst):
            raise ValueError("src and dst must have the same length")
        if not src:
            return
        self._check_ids(src)
        self._check_ids(dst)
        if len(set(dst)) != len(dst) or set(src) & set(dst):
            raise ValueError("copy_blocks needs distinct destinations disjoint from sources")
        n_slots = self.block_size if n_slots is None else int(n_slots)
        s = upload(np.asarray(src, dtype=np.int32), self.device)
        t = upload(np.asarray(dst, dtype=np.int32), self.device)
        if events is not None:
            events[0].record()
        _lib.check(_lib.lib().cx_block_copy(self._pool, s.data_ptr(), t.data_ptr(), len(src),
                                            n_slots, _lib.stream_ptr(self.device)),
                   "cx_block_copy")
        if events is not None:
            events[1].record()

    def compact(self, tables=(), max_moves: int | None = None) -> int:
        """Pack in-use blocks into the lowest ids (``plan_compaction``) and move
        their K/V, every layer, with one ``cx_block_copy``; returns the number
        of blocks moved.  Runs on the cache's current stream, so later kernels
        on that stream see the moved data."""
        src, dst = self.plan_compaction(tables, max_moves)
        if src:
            self.copy_blocks(src, dst)
        return len(src)

    def cow_tail(self, block_table: list, n_tokens: int, is_shared) -> tuple | None:
        """Copy-on-write of a shared, partially filled tail block.

        If position ``n_tokens`` (the next write) falls inside block
        ``block_table[j]`` with ``r = n_tokens % block_size > 0`` valid slots
        and ``is_shared(block_id)`` is true, allocate a private block, copy the
        r valid slots of every layer, and swap it into the table in place.
        Returns (src, dst, r) or None.  The reference has no CoW: it shares
        whole blocks only (radix_kv.py:16-21).
        """
        j, r = divmod(int(n_tokens), self.block_size)
        if r == 0 or j >= len(block_table) or not is_shared(block_table[j]):
            return None
        src = block_table[j]
        dst = self.alloc_block()
        self.copy_blocks([src], [dst], r)
        block_table[j] = dst
        return src, dst, r

    # ------------------------------------------------------------------ #
    # batched forms (many sequences per launch)
    # ------------------------------------------------------------------ #
    def append_batch(self, layer: int, k, v, slot_mapping, cow=None) -> None:
        """k, v: (T, H, D) rows for T tokens of many sequences; slot_mapping:
        (T,) physical slots (``batch.slot_mapping``); optional copy-on-write
        triple (src, dst, n_valid): the first n_valid slots of block src are
        copied into block dst for this layer in the same launch, so no slot
        of the call may fall inside them (checked here for host arrays;
        ``BatchedKVEngine`` builds its slots that way)."""
        if cow is not None:
            _check_cow_slots(slot_mapping, cow, self.block_size)
        kt = to_device(k, self.device)
        vt = to_device(v, self.device)
        st = to_device(slot_mapping, self.device, float_only=False).to(torch.int64)
        if cow is not None:
            cow = tuple(to_device(c, self.device, float_only=False).to(torch.int32) for c in cow)
        self.append_slots(layer, kt, vt, st, cow)

    def append_rope(self, layer: int, k, v, slot_mapping, positions, rope, q=None,
                    q_out_dtype=torch.bfloat16):
        """Rotate K with RoPE while appending it (``apply_rope`` then
        ``write_layer``, transformer.py:84-87), copy V, and return Q rotated
        into a new (T, Hq, D) tensor of ``q_out_dtype`` (None without q).
        k, v: (T, Hkv, D) float32 or bf16; positions: (T,) absolute token
        positions; rope: a ``chenxing_b200.rope.RopeTables``."""
        kt = to_device(k, self.device)
        vt = to_device(v, self.device)
        if kt.dtype not in (torch.float32, torch.bfloat16) or vt.dtype != kt.dtype:
            raise TypeError("k and v must both be float32 or both bfloat16")
        T = int(kt.shape[0])
        shape = (T, self.n_kv_heads, self.head_dim)
        if tuple(kt.shape) != shape or tuple(vt.shape) != shape:
            raise ValueError(f"k/v must have shape {shape}")
        if rope.head_dim != self.head_dim:
            raise ValueError("RoPE tables were built for another head_dim")
        st = to_device(slot_mapping, self.device, float_only=False).to(torch.int64)
        ps = to_device(positions, self.device, float_only=False).to(torch.int64)
        if st.numel() != T or ps.numel() != T:
            raise ValueError("slot_mapping and positions need one entry per token")
        qt = qo = None
        hq = 0
        if q is not None:
            qt = to_device(q, self.device).to(kt.dtype).contiguous()
            if qt.dim() != 3 or qt.shape[0] != T or qt.shape[2] != self.head_dim:
                raise ValueError("q must be (T, Hq, head_dim)")
            hq = int(qt.shape[1])
            qo = torch.empty(tuple(qt.shape), dtype=q_out_dtype, device=self.device)
        _lib.check(_lib.lib().cx_kv_append_rope(
            self._pool, int(layer), kt.contiguous().data_ptr(), vt.contiguous().data_ptr(),
            _lib.cx_dtype(kt.dtype), st.data_ptr(), ps.data_ptr(), T, rope.cos.data_ptr(),
            rope.sin.data_ptr(), rope.rows, int(rope.interleaved), _lib.ptr(qt), hq,
            _lib.ptr(qo), _lib.cx_dtype(q_out_dtype), _lib.stream_ptr(self.device)),
            "cx_kv_append_rope")
        return qo

    def decode_batch(self, layer: int, q, batch, out=None, replan=None):
        """Paged flash-decode of one query token per sequence of ``batch``."""
        from .batch import decode_batch
        return decode_batch(self, layer, q, batch, out, replan)

    def verify_batch(self, layer: int, q, batch, out=None, replan=None):
        """Paged multi-query attention (speculative verify / prefill chunk)."""
        from .batch import verify_batch
        return verify_batch(self, layer, q, batch, out, replan)
