"""Batched KV side of the reference engine's step.

The reference advances its running sequences one at a time
(``ContinuousBatchingScheduler.step``, chenxing/engine/scheduler.py:59-74, over
``LLMEngine.decode_step`` -> ``forward_ids``, chenxing/engine/engine.py:110-168):
per sequence and layer a ``write_layer`` then ``read_layer`` +
``flash_attention``.  ``BatchedKVEngine`` keeps the same per-sequence
metadata rules (prefix hit and acquire at admission, table growth through
``ensure_free`` + ``alloc_block``, ``n_tokens`` as the committed length,
metadata-only rollback, prefix publication and release at finish) and turns
one engine step into ONE ``cx_kv_append`` and ONE paged attention launch per
layer for the whole batch:

    plan = engine.plan([ids...], q_lens)        # host metadata, one H2D
    for layer in range(n_layers):
        engine.append(plan, layer, k, v)        # all sequences' new K/V
        out = engine.attend(plan, layer, q)     # all sequences' queries
    engine.commit(plan)                         # n_tokens += q_len

What the reference does not have and this adds, each opt-in:
* ``add(..., share_tail_from=donor)`` aliases the donor's partially filled
  tail block (the reference shares whole blocks only, radix_kv.py:16-21);
  the first write into an aliased block copies it first (copy-on-write,
  fused into the append launch);
* ``free_private_blocks=True`` returns a finished sequence's private blocks
  to the free list (the reference leaks them, engine.py:98-104);
* ``compact()`` packs in-use blocks into the lowest ids after eviction.
Model projections, sampling and the scheduler's admission policy stay with
the caller.
"""
from __future__ import annotations

from collections import Counter
from dataclasses import dataclass, field

import numpy as np
import torch

from ._arrays import upload
from .batch import PagedBatch, slot_mapping
from .radix_kv import RadixPagedKVCache

__all__ = ["KVSequence", "StepPlan", "BatchedKVEngine"]


@dataclass
class KVSequence:
    """The KV-path fields of the reference ``Sequence`` (sequence.py:20-40)."""
    seq_id: int
    tokens: list                       # Sequence.total_tokens (prompt + generated)
    block_table: list = field(default_factory=list)
    n_tokens: int = 0                  # committed KV positions
    radix_node: object = None
    hit_tokens: int = 0                # positions covered by radix_node's path at admission
    aliased: set = field(default_factory=set)   # table indices shared by add(share_tail_from)


@dataclass
class StepPlan:
    """Metadata of one engine step for a batch of sequences."""
    seqs: list
    n_past: np.ndarray                 # committed positions before the step
    q_lens: np.ndarray
    batch: PagedBatch | None           # None for write-only steps
    slots: torch.Tensor | None         # (sum q_lens,) int64 physical slots
    cow: tuple | None                  # (src, dst, n_valid) int32 device tensors
    cow_host: list                     # [(src, dst, n_valid)]
    appended: set = field(default_factory=set)
    positions: torch.Tensor | None = None   # (sum q_lens,) absolute positions, built lazily
    cow_done: bool = False

    @property
    def n_rows(self) -> int:
        return int(self.q_lens.sum())


class BatchedKVEngine:
    """Owns the live sequences' block tables over one ``RadixPagedKVCache``."""

    def __init__(self, cache: RadixPagedKVCache, *, n_q_heads: int, window: int | None = None,
                 scale: float | None = None, free_private_blocks: bool = False,
                 publish_mode: str = "reference") -> None:
        if publish_mode not in ("reference", "suffix"):
            raise ValueError("publish_mode must be 'reference' or 'suffix'")
        self.cache = cache
        self.publish_mode = publish_mode
        self.n_q_heads = int(n_q_heads)
        self.window = window
        self.scale = scale
        self.free_private_blocks = free_private_blocks
        self.seqs: dict = {}
        self._alias_refs: Counter = Counter()     # block id -> live sequences aliasing it
        self._held: Counter = Counter()           # block id -> live tables listing it

    # ------------------------------------------------------------------ #
    # admission / lifecycle
    # ------------------------------------------------------------------ #
    def add(self, seq_id: int, prompt_tokens: list, *, share_tail_from: int | None = None
            ) -> KVSequence:
        """Admit a sequence: longest cached prefix, zero-copy, pinned
        (``LLMEngine.prefill``, engine.py:140-147).  A full prompt hit leaves
        the last prompt token to be re-forwarded, as the reference does
        (engine.py:152-156).  ``share_tail_from`` additionally aliases a live
        donor's partially filled block that follows the hit, when the donor
        has committed those positions with the same tokens."""
        if seq_id in self.seqs:
            raise ValueError(f"sequence {seq_id} already live")
        if not prompt_tokens:
            raise ValueError("prompt must contain at least one token")
        c = self.cache
        s = KVSequence(seq_id, list(prompt_tokens))
        hit = c.match_prefix(s.tokens)
        s.block_table = list(hit.block_ids)
        if hit.n_tokens > 0:
            c.acquire(hit.node)
            s.radix_node = hit.node
        s.n_tokens = s.hit_tokens = hit.n_tokens
        if share_tail_from is not None:
            d = self.seqs[share_tail_from]
            j = len(s.block_table)
            r = min(d.n_tokens - hit.n_tokens, c.block_size - 1,
                    len(s.tokens) - hit.n_tokens)
            if (r > 0 and d.block_table[:j] == s.block_table and len(d.block_table) > j
                    and d.tokens[hit.n_tokens:hit.n_tokens + r]
                    == s.tokens[hit.n_tokens:hit.n_tokens + r]):
                b = d.block_table[j]
                s.block_table.append(b)
                s.n_tokens += r
                s.aliased.add(j)
                if j not in d.aliased:
                    d.aliased.add(j)
                    self._alias_refs[b] += 1
                self._alias_refs[b] += 1
        if s.n_tokens == len(s.tokens):
            s.n_tokens -= 1
        self.seqs[seq_id] = s
        self._held.update(s.block_table)
        return s

    def finish(self, seq_id: int, publish: bool = True) -> None:
        """Publish the block-aligned committed prefix into the radix tree and
        unpin (``_publish_prefix`` + ``_release_seq``, engine.py:98-104,
        192-204).  With ``free_private_blocks`` the blocks the tree did not
        take over go back to the free list."""
        c = self.cache
        if publish:
            self.publish(seq_id)
        s = self.seqs.pop(seq_id)
        if s.radix_node is not None:
            try:
                c.release(s.radix_node)
            except RuntimeError:
                pass
            s.radix_node = None
        for j in s.aliased:
            b = s.block_table[j]
            self._alias_refs[b] -= 1
            if self._alias_refs[b] <= 0:
                del self._alias_refs[b]
        self._unhold(s.block_table)
        if self.free_private_blocks:
            # blocks no radix node and no other live table lists
            held = self._held
            c._free_blocks([b for b in s.block_table if not c.tree_holds(b) and b not in held])

    def publish(self, seq_id: int) -> bool:
        """Insert the block-aligned committed prefix into the radix tree under
        the sequence's hit node (``_publish_prefix``, engine.py:192-204); the
        sequence stays live.  Returns whether anything was inserted.

        ``publish_mode="reference"`` inserts the whole chain from token 0
        under the hit node, as the reference does: the new node aliases the
        hit path's blocks, and evicting it later frees blocks that the hit
        path and the sequences pinning it still use (they are then handed
        out again and overwritten).  ``"suffix"`` inserts only the part past
        the hit, which keeps one owner per block."""
        c = self.cache
        s = self.seqs[seq_id]
        bs = c.block_size
        full = s.n_tokens // bs
        skip = s.hit_tokens // bs if (self.publish_mode == "suffix" and s.radix_node) else 0
        if full <= skip:
            return False
        try:
            c.insert(s.tokens[skip * bs:full * bs], s.block_table[skip:full], parent=s.radix_node)
        except ValueError:
            return False
        return True

    def rollback(self, seq_id: int, n_target: int) -> None:
        """Metadata-only shrink (``SpeculativeDecoder._sync_to``,
        speculative.py:86-92): the table keeps its blocks."""
        s = self.seqs[seq_id]
        if s.n_tokens > n_target:
            s.n_tokens = int(n_target)

    def extend_tokens(self, seq_id: int, new_tokens: list) -> None:
        """Append generated / drafted token ids (Sequence.generated)."""
        self.seqs[seq_id].tokens.extend(int(t) for t in new_tokens)

    def _unhold(self, blocks) -> None:
        self._held.subtract(blocks)
        for b in blocks:
            if self._held[b] <= 0:
                del self._held[b]

    # ------------------------------------------------------------------ #
    # one step
    # ------------------------------------------------------------------ #
    def plan(self, seq_ids, q_lens=None, *, verify: bool | None = None,
             attend: bool = True) -> StepPlan:
        """Host metadata for one step: ``q_lens[i]`` new positions for
        sequence ``seq_ids[i]`` starting at its ``n_tokens``.  Grows tables like
        ``LLMEngine._ensure_capacity`` (engine.py:74-85, LRU eviction through
        ``ensure_free``; ``OutOfKVCacheError`` is left to the scheduler's
        preemption policy), privatises aliased blocks about to be written,
        and loads the batch's slots (and, with ``attend``, tables and
        lengths) onto the device.  ``attend=False`` is for steps that only
        write K/V (a prompt whose attention the caller does elsewhere)."""
        p = self.plan_host(seq_ids, q_lens)
        c = self.cache
        dev = c.device
        bs = c.block_size
        p.slots = upload(slot_mapping([s.block_table for s in p.seqs], p.n_past, p.q_lens, bs),
                         dev)
        if attend:
            is_verify = bool(np.any(p.q_lens != 1)) if verify is None else verify
            p.batch = PagedBatch(c, [s.block_table for s in p.seqs], p.n_past + p.q_lens,
                                 n_q_heads=self.n_q_heads,
                                 q_lens=p.q_lens if is_verify else None,
                                 window=self.window, scale=self.scale)
        if p.cow_host:
            arr = np.asarray(p.cow_host, dtype=np.int32).T.copy()
            p.cow = tuple(upload(a, dev) for a in arr)
        return p

    def plan_host(self, seq_ids, q_lens=None) -> StepPlan:
        """The host half of ``plan``: table growth and copy-on-write choices
        only (no device arrays); also usable over a bare ``RadixIndex``."""
        c = self.cache
        bs = c.block_size
        seqs = [self.seqs[i] for i in seq_ids]
        ql = np.ones(len(seqs), dtype=np.int64) if q_lens is None else \
            np.asarray(q_lens, dtype=np.int64).reshape(-1)
        if ql.shape[0] != len(seqs) or np.any(ql < 0):
            raise ValueError("q_lens must give a non-negative count per sequence")
        n_past = np.array([s.n_tokens for s in seqs], dtype=np.int64)
        cow = []
        for s, n in zip(seqs, ql):
            if n == 0:
                continue
            first, last = s.n_tokens // bs, (s.n_tokens + int(n) - 1) // bs
            for j in sorted(s.aliased):
                if first <= j <= last:
                    src = s.block_table[j]
                    if self._alias_refs[src] > 1:
                        c.ensure_free(1)
                        dst = c.alloc_block()
                        cow.append((src, dst, s.n_tokens - j * bs if j == first else 0))
                        s.block_table[j] = dst
                        self._unhold([src])
                        self._held[dst] += 1
                    self._alias_refs[src] -= 1
                    if self._alias_refs[src] <= 0:
                        del self._alias_refs[src]
                    s.aliased.discard(j)
            target = s.n_tokens + int(n)
            have = len(s.block_table) * bs
            if target > have:
                need = -(-(target - have) // bs)
                c.ensure_free(need)
                new = c.alloc_blocks(need)
                s.block_table.extend(new)
                self._held.update(new)
        return StepPlan(seqs, n_past, ql, None, None, None, cow)

    def append(self, plan: StepPlan, layer: int, k, v) -> None:
        """Write the step's new K/V rows (sum q_lens, Hkv, D) of one layer, with
        the plan's copy-on-write copies of that layer fused in."""
        self.cache.append_batch(layer, k, v, plan.slots, cow=plan.cow)
        plan.appended.add(int(layer))

    def append_rope(self, plan: StepPlan, layer: int, k, v, rope, q=None,
                    q_out_dtype=torch.bfloat16):
        """``append`` with RoPE fused in: K rotated at each token's absolute
        position (its sequence's committed length + index in the step), V
        copied, and Q rotated into the returned tensor (transformer.py:84-87).
        The plan's copy-on-write copies run once, for every layer, before the
        first such call."""
        if plan.cow_host and not plan.cow_done:
            for src, dst, n in plan.cow_host:          # all layers at once
                if n > 0:
                    self.cache.copy_blocks([src], [dst], n)
            plan.cow_done = True
        if plan.positions is None:
            pos = np.concatenate([np.arange(n0, n0 + n, dtype=np.int64)
                                  for n0, n in zip(plan.n_past, plan.q_lens)]) \
                if len(plan.q_lens) else np.zeros(0, dtype=np.int64)
            plan.positions = upload(pos, self.cache.device)
        qo = self.cache.append_rope(layer, k, v, plan.slots, plan.positions, rope, q,
                                    q_out_dtype)
        plan.appended.add(int(layer))
        return qo

    def attend(self, plan: StepPlan, layer: int, q, out=None):
        """Paged attention of the step's query rows (sum q_lens, Hq, D) over
        every committed position plus the step's own; float32 output."""
        if plan.batch is None:
            raise RuntimeError("plan(..., attend=False) has no attention batch")
        if int(layer) not in plan.appended:
            raise RuntimeError("attend() before append() for this layer: the step's own "
                               "keys would be missing")
        if plan.batch.verify:
            return self.cache.verify_batch(layer, q, plan.batch, out)
        return self.cache.decode_batch(layer, q, plan.batch, out)

    def commit(self, plan: StepPlan) -> None:
        """``forward_ids``'s ``seq.n_tokens += len(new_ids)`` (engine.py:127)."""
        for s, n in zip(plan.seqs, plan.q_lens):
            s.n_tokens += int(n)

    # ------------------------------------------------------------------ #
    def compact(self, max_moves: int | None = None, events=None) -> int:
        """Pack in-use blocks into the lowest ids (every live table and the
        radix tree are relabelled, the K/V moved by one block-copy launch);
        returns blocks moved.  ``events``: optional pair of CUDA events
        recorded around the copy launch (when there is one)."""
        live = [s.block_table for s in self.seqs.values()]
        src, dst = self.cache.plan_compaction(live, max_moves)
        if src and isinstance(self.cache, RadixPagedKVCache):
            self.cache.copy_blocks(src, dst, events=events)   # bare RadixIndex: metadata only
        n = len(src)
        for a, b in zip(src, dst):
            if a in self._held:
                self._held[b] += self._held.pop(a)
        if n and self._alias_refs:
            refs = Counter()
            for s in self.seqs.values():
                for j in s.aliased:
                    refs[s.block_table[j]] += 1
            self._alias_refs = refs
        return n
