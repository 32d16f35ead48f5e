"""Oracle replay of the batched engine's metadata policy — TEST INFRASTRUCTURE.

Restates, one sequence at a time on the oracle cache (``oracle.radix_kv``,
metadata only), what ``chenxing_b200.engine.BatchedKVEngine`` must do to the
block tables, free list and radix tree:

* admission = ``LLMEngine.prefill``'s prefix part (chenxing/engine/engine.py:140-147,
  152-156): match, take the hit blocks, acquire, full hit -> re-forward the
  last prompt token;
* a step    = ``forward_ids`` per sequence in batch order (engine.py:110-129):
  ``_ensure_capacity`` (engine.py:74-85), then ``n_tokens += q_len``;
* finish    = ``_publish_prefix`` then ``_release_seq`` (engine.py:98-104,
  192-204), plus, when asked, freeing the blocks neither the tree nor a live
  sequence holds (the reference leaks them).  ``suffix_publish`` restates the
  corrected publication: only the chain past the hit goes under the hit node;
* compaction = ``oracle.paged.compact``.
"""
from __future__ import annotations

from oracle.paged import compact, ensure_capacity


class OracleEngine:
    def __init__(self, meta, free_private=False, suffix_publish=False):
        self.meta = meta
        self.free_private = free_private
        self.suffix_publish = suffix_publish
        self.seqs = {}

    def add(self, sid, prompt):
        m = self.meta
        hit = m.match_prefix(prompt)
        s = {"tokens": list(prompt), "table": list(hit.block_ids), "n": hit.n_tokens,
             "node": None, "hit": hit.n_tokens}
        if hit.n_tokens > 0:
            m.acquire(hit.node)
            s["node"] = hit.node
        if s["n"] == len(prompt):
            s["n"] -= 1
        self.seqs[sid] = s
        return s

    def step(self, ids, q_lens):
        for sid, q in zip(ids, q_lens):
            s = self.seqs[sid]
            if q:
                ensure_capacity(self.meta, s["table"], s["n"] + int(q))

    def commit(self, ids, q_lens):
        for sid, q in zip(ids, q_lens):
            self.seqs[sid]["n"] += int(q)

    def _tree_blocks(self):
        out, todo = set(), [self.meta._root]
        while todo:
            n = todo.pop()
            out |= set(n.blocks)
            todo += list(n.children.values())
        return out

    def finish(self, sid, publish=True):
        m = self.meta
        s = self.seqs.pop(sid)
        bs = m.block_size
        full = s["n"] // bs
        lo = s["hit"] // bs if (self.suffix_publish and s["node"] is not None) else 0
        if publish and full > lo:
            try:
                m.insert(s["tokens"][lo * bs:full * bs], s["table"][lo:full], parent=s["node"])
            except ValueError:
                pass
        if s["node"] is not None:
            try:
                m.release(s["node"])
            except RuntimeError:
                pass
        if self.free_private:
            keep = self._tree_blocks()
            for o in self.seqs.values():
                keep |= set(o["table"])
            for b in s["table"]:
                if b not in keep:
                    m._free_block(b)

    def compact(self, max_moves=None):
        return compact(self.meta, [s["table"] for s in self.seqs.values()], max_moves)
