"""Per-sequence paged decode / verify oracle — TEST INFRASTRUCTURE ONLY.

Restates how the reference drives the KV hot path, one sequence at a time:

* ``attend_sequence``  — ``Transformer.forward`` per layer
  (``chenxing/model/transformer.py:87-94``): ``write_layer`` at ``n_past``,
  ``read_layer`` of ``n_past + T`` tokens, transpose to (1, h, T, d), then
  ``flash_attention(q4, k4, v4, CausalMask())``.  Windowed cases use
  ``naive_attention`` (``chenxing/core/attention.py:119``) because the blocked
  kernel returns NaN when a leading key block is fully masked.
* ``ensure_capacity`` — ``LLMEngine._ensure_capacity`` (``chenxing/engine/engine.py:74-85``),
  block-table growth through ``ensure_free`` + ``alloc_block``.
* ``rollback``        — ``SpeculativeDecoder._sync_to`` shrink branch
  (``chenxing/engine/speculative.py:86-92``): metadata-only, table untouched.
* ``slot_mapping``    — the token -> physical slot rule of ``write_layer``
  (``chenxing/engine/radix_kv.py:123-128``): ``bt[p // bs] * bs + p % bs``.
* ``cow_tail``        — copy-on-write of a shared partial tail block.  The
  reference has no CoW (it shares whole blocks only, ``radix_kv.py:16-21``);
  this oracle defines it by construction: take ``alloc_block()``, copy the
  ``r = n_tokens % bs`` valid slots of every layer, swap the table entry.
* ``compact``         — block-pool compaction after eviction; also absent from
  the reference (it never moves data).  Defined by construction: two
  pointers, the lowest free id below ``n_used`` and the highest in-use id at
  or above it, are paired until they cross; data copied, radix nodes and
  tables relabelled, vacated ids appended to the free list in ascending order.
"""
from __future__ import annotations

import numpy as np

from .attention import CausalMask, flash_attention, naive_attention

__all__ = ["slot_mapping", "ensure_capacity", "rollback", "cow_tail", "compact",
           "attend_sequence", "paged_attention_batch"]


def slot_mapping(block_table, start, n, block_size):
    pos = np.arange(start, start + n, dtype=np.int64)
    bt = np.asarray(block_table, dtype=np.int64)
    return bt[pos // block_size] * block_size + pos % block_size


def ensure_capacity(cache, block_table, target_tokens):
    """Grow ``block_table`` in place so it covers ``target_tokens`` positions."""
    have = len(block_table) * cache.block_size
    if target_tokens <= have:
        return
    need = -(-(target_tokens - have) // cache.block_size)
    cache.ensure_free(need)
    for _ in range(need):
        block_table.append(cache.alloc_block())


def rollback(n_tokens, n_target):
    """Speculative rollback: shrink the committed length, keep the table."""
    return n_target if n_tokens > n_target else n_tokens


def cow_tail(cache, block_table, n_tokens, is_shared):
    """Privatise the block that position ``n_tokens`` falls in, if shared.

    Returns ``(src, dst, n_valid)`` when a copy was made, else ``None``.
    """
    bs = cache.block_size
    j = n_tokens // bs
    r = n_tokens % bs
    if r == 0 or j >= len(block_table) or not is_shared(block_table[j]):
        return None
    src = block_table[j]
    dst = cache.alloc_block()
    cache.k_pool[:, dst, :r] = cache.k_pool[:, src, :r]
    cache.v_pool[:, dst, :r] = cache.v_pool[:, src, :r]
    block_table[j] = dst
    return src, dst, r


def compact(cache, tables, max_moves=None):
    """Pack in-use blocks into the lowest ids; returns the (src, dst) moves."""
    free = cache._free
    n_used = cache.n_blocks - len(free)
    lo, hi, moves = 0, cache.n_blocks - 1, []
    while max_moves is None or len(moves) < max_moves:
        while lo < n_used and lo not in free:
            lo += 1
        while hi >= n_used and hi in free:
            hi -= 1
        if lo >= n_used or hi < n_used:
            break
        moves.append((hi, lo))
        lo, hi = lo + 1, hi - 1
    if not moves:
        return []
    if hasattr(cache, "k_pool"):
        for s, d in moves:
            cache.k_pool[:, d] = cache.k_pool[:, s]
            cache.v_pool[:, d] = cache.v_pool[:, s]
    new_id = dict(moves)
    todo = [cache._root]
    while todo:
        node = todo.pop()
        node.blocks = [new_id.get(b, b) for b in node.blocks]
        todo.extend(node.children.values())
    for t in tables:
        for i, b in enumerate(t):
            if b in new_id:
                t[i] = new_id[b]
    for _, d in moves:
        del free[d]
    for s in sorted(s for s, _ in moves):
        free[s] = None
    return moves


def attend_sequence(cache, block_table, n_past, layer, q, k_new, v_new,
                    window=None, scale=None, write=True):
    """One sequence, one layer: append T tokens then attend over n_past+T keys.

    q (T, hq, d); k_new / v_new (T, hkv, d).  Returns float32 (T, hq, d).
    """
    t = q.shape[0]
    if write:
        cache.write_layer(block_table, n_past, layer, k_new, v_new)
    k_all, v_all = cache.read_layer(block_table, n_past + t, layer)
    q4 = np.ascontiguousarray(np.transpose(q, (1, 0, 2))[None])
    k4 = np.ascontiguousarray(np.transpose(k_all, (1, 0, 2))[None])
    v4 = np.ascontiguousarray(np.transpose(v_all, (1, 0, 2))[None])
    if window is None:
        o = flash_attention(q4, k4, v4, CausalMask(), scale)
    else:
        o = naive_attention(q4, k4, v4, CausalMask(window), scale)
    return np.ascontiguousarray(o[0].transpose(1, 0, 2))


def paged_attention_batch(cache, layer, q, block_tables, ctx_lens, q_lens,
                          window=None, scale=None):
    """Attention for a batch of sequences whose new K/V are already written.

    q (sum(q_lens), hq, d) token-major; sequence b's rows are the last
    ``q_lens[b]`` positions of its ``ctx_lens[b]`` cached tokens.
    """
    outs, r = [], 0
    for bt, ctx, ql in zip(block_tables, ctx_lens, q_lens):
        qb = q[r:r + ql]
        r += ql
        if ctx == 0:
            outs.append(np.zeros((ql,) + q.shape[1:], dtype=np.float32))
            continue
        outs.append(attend_sequence(cache, bt, ctx - ql, layer, qb, None, None,
                                    window=window, scale=scale, write=False))
    if not outs:
        return np.zeros((0,) + q.shape[1:], dtype=np.float32)
    return np.concatenate(outs, axis=0)
