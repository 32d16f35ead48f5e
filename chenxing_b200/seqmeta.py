"""Per-sequence block-table metadata rules of the reference engine.

These stay host-side Python, exactly as the reference does them, so the
batched GPU path sees the same block tables and lengths:

* ``grow_table`` — ``LLMEngine._ensure_capacity`` (chenxing/engine/engine.py:74-85):
  append ``ceil((target - have) / bs)`` blocks from the FIFO free list after
  ``ensure_free`` (LRU eviction).  Preemption is the caller's policy.
* ``rollback``   — ``SpeculativeDecoder._sync_to`` shrink branch
  (chenxing/engine/speculative.py:86-92): O(1), metadata only; the block
  table keeps the blocks of rejected drafts and the next forward overwrites
  their stale slots.
"""
from __future__ import annotations

__all__ = ["grow_table", "rollback"]


def grow_table(index, block_table: list, target_tokens: int) -> int:
    """Grow ``block_table`` in place to cover ``target_tokens`` positions;
    returns the number of blocks appended."""
    have = len(block_table) * index.block_size
    if target_tokens <= have:
        return 0
    need = -(-(target_tokens - have) // index.block_size)
    index.ensure_free(need)
    for _ in range(need):
        block_table.append(index.alloc_block())
    return need


def rollback(n_tokens: int, n_target: int) -> int:
    """Committed length after a speculative rollback to ``n_target``."""
    return n_target if n_tokens > n_target else n_tokens
