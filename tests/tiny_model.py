"""The reference's tiny decoder around a pluggable KV cache — TEST INFRASTRUCTURE.

Drives the KV hot path the way the reference's model and engine do, so that
the drop-ins (``chenxing_b200.RadixPagedKVCache`` and
``chenxing_b200.flash_attention``) can be checked inside the reference's own
end-to-end invariants with the reference's own weights
(``tests/golden/tiny_model.npz``, written by ``make_golden.py``):

* ``TinyDecoder.forward`` restates ``Transformer.forward``
  (chenxing/model/transformer.py:65-104): pre-norm RMSNorm, rotary
  embeddings, grouped-query attention, SwiGLU FFN, in NumPy float32; per
  layer exactly the reference's KV calls — ``write_layer`` at ``n_past``,
  ``read_layer`` of ``n_past + T`` tokens, ``flash_attention(q4, k4, v4,
  CausalMask())`` on (1, h, T, d) arrays;
* ``TinyEngine`` restates ``LLMEngine.prefill / forward_ids / generate``
  (chenxing/engine/engine.py:74-85, 110-190) for greedy decoding;
* ``speculative_greedy`` restates the greedy branch of
  ``SpeculativeDecoder.generate`` (chenxing/engine/speculative.py:86-200):
  draft gamma tokens, verify them with one target forward of gamma + 1
  tokens, metadata-only rollback of ``n_tokens``.

The cache class and the attention function are parameters: the oracle pair
pins this restatement to the goldens on the CPU, the product pair runs it on
the GPU.
"""
from __future__ import annotations

import numpy as np

from oracle.rope import rope_tables, rotate


class TinyDecoder:
    def __init__(self, g, tag: str, flash_attention, CausalMask):
        vocab, hidden, inter, layers, hq, hk, hd = (int(x) for x in g[f"{tag}.config"])
        theta, eps, max_pos = (float(x) for x in g[f"{tag}.rope"])
        self.vocab, self.hq, self.hk, self.hd, self.eps = vocab, hq, hk, hd, eps
        self.n_layers = layers
        w = {k[len(tag) + 1:]: g[k] for k in g.files if k.startswith(tag + ".blk.")
             or k in (f"{tag}.token_embd.weight", f"{tag}.output_norm.weight",
                      f"{tag}.output.weight")}
        self.emb = w["token_embd.weight"]
        self.out_norm = w["output_norm.weight"]
        self.out_w = w.get("output.weight", self.emb)
        self.layers = [{n: w[f"blk.{i}.{n}.weight"] for n in
                        ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                         "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")}
                       for i in range(layers)]
        self.cos, self.sin = rope_tables(int(max_pos), hd, theta)
        self.flash, self.mask = flash_attention, CausalMask

    def _norm(self, x, w):
        return x * (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + self.eps)) * w

    def forward(self, ids, positions, kv, block_table, n_past):
        ids = np.asarray(ids, dtype=np.int64)
        x = self.emb[ids]
        total = n_past + len(ids)
        for li, L in enumerate(self.layers):
            h = self._norm(x, L["attn_norm"])
            q = (h @ L["attn_q"].T).reshape(-1, self.hq, self.hd)
            k = (h @ L["attn_k"].T).reshape(-1, self.hk, self.hd)
            v = (h @ L["attn_v"].T).reshape(-1, self.hk, self.hd)
            q = rotate(q, self.cos, self.sin, positions)
            k = rotate(k, self.cos, self.sin, positions)
            kv.write_layer(block_table, n_past, li, k, v)
            k_all, v_all = kv.read_layer(block_table, total, li)
            q4 = np.ascontiguousarray(np.transpose(q, (1, 0, 2))[None])
            k4 = np.ascontiguousarray(np.transpose(np.asarray(k_all, np.float32), (1, 0, 2))[None])
            v4 = np.ascontiguousarray(np.transpose(np.asarray(v_all, np.float32), (1, 0, 2))[None])
            a = np.asarray(self.flash(q4, k4, v4, self.mask()))[0]
            x = x + a.transpose(1, 0, 2).reshape(len(ids), -1) @ L["attn_output"].T
            h = self._norm(x, L["ffn_norm"])
            gate = h @ L["ffn_gate"].T
            x = x + ((gate / (1.0 + np.exp(-gate))) * (h @ L["ffn_up"].T)) @ L["ffn_down"].T
        return self._norm(x, self.out_norm) @ self.out_w.T


class TinySeq:
    def __init__(self, tokens):
        self.tokens = list(tokens)
        self.block_table: list = []
        self.n_tokens = 0
        self.node = None


class TinyEngine:
    """Greedy engine over one cache: block size 8, 64 blocks, as the
    reference's test engines."""

    def __init__(self, model: TinyDecoder, make_cache):
        self.model = model
        self.kv = make_cache(64, 8, model.n_layers, model.hk, model.hd)

    def _ensure_capacity(self, seq, target):
        have = len(seq.block_table) * self.kv.block_size
        if target > have:
            need = -(-(target - have) // self.kv.block_size)
            self.kv.ensure_free(need)
            for _ in range(need):
                seq.block_table.append(self.kv.alloc_block())

    def forward_ids(self, seq, ids):
        n_past = seq.n_tokens
        self._ensure_capacity(seq, n_past + len(ids))
        pos = np.arange(n_past, n_past + len(ids), dtype=np.int64)
        logits = self.model.forward(ids, pos, self.kv, seq.block_table, n_past)
        seq.n_tokens += len(ids)
        return logits

    def prefill(self, seq, prompt):
        hit = self.kv.match_prefix(prompt)
        seq.block_table = list(hit.block_ids)
        if hit.n_tokens > 0:
            self.kv.acquire(hit.node)
            seq.node = hit.node
        rest = prompt[hit.n_tokens:]
        if rest:
            seq.n_tokens = hit.n_tokens
            return self.forward_ids(seq, rest)[-1]
        seq.n_tokens = hit.n_tokens - 1
        return self.forward_ids(seq, prompt[-1:])[-1]

    def generate_greedy(self, prompt, max_tokens):
        seq = TinySeq(prompt)
        logits = self.prefill(seq, list(prompt))
        out = []
        while len(out) < max_tokens:
            if seq.n_tokens < len(seq.tokens):
                logits = self.forward_ids(seq, seq.tokens[seq.n_tokens:seq.n_tokens + 1])[-1]
            tok = int(np.argmax(logits))
            out.append(tok)
            seq.tokens.append(tok)
        return out


def speculative_greedy(target: TinyEngine, draft: TinyEngine, prompt, gamma, max_tokens):
    """Greedy speculative decoding; returns (tokens, [steps, drafted, accepted])."""
    tseq, dseq = TinySeq(prompt), TinySeq(prompt)
    target.prefill(tseq, list(prompt))
    draft.prefill(dseq, list(prompt))
    confirmed = list(prompt)
    tseq.n_tokens -= 1
    dseq.n_tokens -= 1
    steps = drafted = accepted = 0

    def sync(seq, eng, n_target):
        if seq.n_tokens > n_target:
            seq.n_tokens = n_target                   # metadata-only rollback
        elif seq.n_tokens < n_target:
            eng.forward_ids(seq, confirmed[seq.n_tokens:n_target])

    while len(confirmed) - len(prompt) < max_tokens:
        n_start = len(confirmed) - 1
        sync(dseq, draft, n_start)
        proposed = []
        row = draft.forward_ids(dseq, [confirmed[n_start]])[-1]
        for i in range(gamma):
            tok = int(np.argmax(row))
            proposed.append(tok)
            drafted += 1
            if i < gamma - 1:
                row = draft.forward_ids(dseq, [tok])[-1]
        sync(tseq, target, n_start)
        logits = target.forward_ids(tseq, [confirmed[n_start]] + proposed)
        n_ok, nxt = 0, None
        for i, tok in enumerate(proposed):
            if tok == int(np.argmax(logits[i])):
                n_ok += 1
                continue
            nxt = int(np.argmax(logits[i]))
            break
        else:
            nxt = int(np.argmax(logits[-1]))
        accepted += n_ok
        steps += 1
        confirmed.extend(proposed[:n_ok])
        confirmed.append(nxt)
        if n_ok < gamma:
            n_target = len(confirmed) - 1
            sync(dseq, draft, n_target)
            sync(tseq, target, n_target)
    return confirmed[len(prompt):][:max_tokens], [steps, drafted, accepted]
