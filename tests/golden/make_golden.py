"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Usage (needs a checkout of the reference Chenxing repo; it is pure NumPy):

    python tests/golden/make_golden.py --reference <path-to-chenxing-checkout>

Writes:
  attention.npz   reference flash/naive attention outputs for the reference's
                  own test shapes plus decode / verify / window / bf16 / dv!=d
                  / explicit-mask cases; inputs are rebuilt from cases.py and
                  pinned by the digests in attention_cases.json.
  paged_cfg1.npz  the cfg1 decode run driven through the reference
                  RadixPagedKVCache.write_layer -> read_layer -> flash_attention
                  (chenxing/model/transformer.py:87-94), outputs at a few steps
                  and a digest of the seeded inputs.
  paged_bf16.npz  a cfg2-shaped bf16 (ml_dtypes) pool, one decode step
                  (inputs from cases.paged_bf16_inputs, pinned by digest).
  radix_ops.json  a seeded script of pool / radix-tree operations replayed on
                  the reference with a logical LRU clock, with every result.
  engine_meta.json block-table growth (LLMEngine._ensure_capacity), speculative
                  rollback (SpeculativeDecoder._sync_to) and the slot each
                  written token landed in, observed from the reference pool.
  rope.npz        reference build_rope_cache tables (plain and YaRN-scaled) and
                  apply_rope outputs (half-split and interleaved layouts, token
                  positions picked from the table) on seeded inputs.
  tiny_model.npz  the reference's own tiny seeded target and draft models
                  (tests/conftest.py of the reference) run through its
                  LLMEngine and SpeculativeDecoder: their weights, the logits
                  of the full / incremental / rollback-and-rewrite prefills of
                  its tests/test_transformer.py:7-23, and the greedy target
                  and speculative (gamma 1, 2, 4, 8) outputs of its
                  tests/test_speculative.py:14-21.

    python tests/golden/make_golden.py --reference <path> --only rope
    python tests/golden/make_golden.py --reference <path> --only model

regenerate rope.npz / tiny_model.npz alone.
"""
from __future__ import annotations

import argparse
import hashlib
import itertools
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def attention_outputs(ref_attn, CausalMask):
    from cases import attention_cases, case_digest
    out, meta = {}, []
    for c in attention_cases():
        if c["mask"] == "causal":
            m = CausalMask(sliding_window=c["window"])
        elif c["mask"] == "explicit":
            m = c["explicit"]
        else:
            m = None
        fn = ref_attn.flash_attention if c["use"] == "flash" else ref_attn.naive_attention
        out[c["name"]] = fn(c["q"], c["k"], c["v"], m, c["scale"])
        meta.append({"name": c["name"], "digest": case_digest(c)})
    return out, meta


def paged_cfg1(RadixPagedKVCache, flash, CausalMask):
    from chenxing_b200.workloads import cfg1
    wl, data = cfg1(seed=0)
    cache = RadixPagedKVCache(wl.n_blocks, wl.block_size, 1, wl.n_kv_heads,
                              wl.head_dim, dtype=np.float32)
    ctx = wl.ctx_lens.copy()
    for b in range(wl.batch):
        cache.write_layer(wl.block_tables[b], 0, 0, data["k_pre"][b], data["v_pre"][b])
    keep = [0, 1, 15, 31]
    res = {}
    for s in range(wl.steps):
        outs = []
        for b in range(wl.batch):
            bt = wl.block_tables[b]
            cache.write_layer(bt, int(ctx[b]), 0, data["k"][s, b][None], data["v"][s, b][None])
            ka, va = cache.read_layer(bt, int(ctx[b]) + 1, 0)
            q4 = data["q"][s, b][:, None, :][None]                       # (1, hq, 1, d)
            k4 = np.ascontiguousarray(np.transpose(ka, (1, 0, 2))[None])
            v4 = np.ascontiguousarray(np.transpose(va, (1, 0, 2))[None])
            outs.append(flash(q4, k4, v4, CausalMask())[0][:, 0, :])     # (hq, d)
            ctx[b] += 1
        if s in keep:
            res[f"out_step{s}"] = np.stack(outs)
    res["final_ctx"] = ctx
    res["input_digest"] = np.frombuffer(
        digest(wl.ctx_lens, np.asarray(sum(wl.block_tables, [])),
               *data["k_pre"], *data["v_pre"], data["q"], data["k"], data["v"]).encode(),
        dtype=np.uint8)
    res["pool_digest"] = np.frombuffer(digest(cache.k_pool, cache.v_pool).encode(),
                                       dtype=np.uint8)
    return res


def paged_bf16(RadixPagedKVCache, flash, CausalMask, bf16):
    from cases import paged_bf16_inputs
    wl, ks, vs, qs = paged_bf16_inputs()
    cache = RadixPagedKVCache(wl.n_blocks, wl.block_size, 1, wl.n_kv_heads,
                              wl.head_dim, dtype=bf16)
    outs, bits = [], []
    for b in range(wl.batch):
        c = int(wl.ctx_lens[b]) + 1
        cache.write_layer(wl.block_tables[b], 0, 0, ks[b], vs[b])
        ka, va = cache.read_layer(wl.block_tables[b], c, 0)
        q4 = qs[b][:, None, :][None]
        k4 = np.ascontiguousarray(np.transpose(ka, (1, 0, 2))[None])
        v4 = np.ascontiguousarray(np.transpose(va, (1, 0, 2))[None])
        outs.append(flash(q4, k4, v4, CausalMask())[0][:, 0, :])
        bits.append(ka.view(np.uint16))
    return {"out": np.stack(outs),
            "input_digest": np.frombuffer(digest(*ks, *vs, *qs).encode(), dtype=np.uint8),
            "kbits_digest": np.frombuffer(digest(*bits).encode(), dtype=np.uint8)}


def radix_script(ref_radix, n_ops=700, seed=5):
    """Seeded request-driven workload over the reference cache.

    Requests draw prompts from a few shared documents so prefixes hit; each
    op and its result (block ids, hit lengths, node handles, freed counts,
    error class, FIFO free-list order, stats) is recorded for replay.
    """
    clock = itertools.count()
    ref_radix.time.monotonic = lambda: float(next(clock))
    bs = 4
    cache = ref_radix.RadixPagedKVCache(n_blocks=40, block_size=bs, n_layers=1,
                                        n_kv_heads=1, head_dim=2)
    rng = np.random.default_rng(seed)
    docs = [[int(t) for t in rng.integers(0, 6, 28)] for _ in range(5)]
    handles = [None]          # handle 0 = "no node"
    pinned = []
    ops = []
    last_hit = {"blocks": [], "node": 0, "tokens": []}

    def h_of(node):
        for i, n in enumerate(handles):
            if n is node:
                return i
        handles.append(node)
        return len(handles) - 1

    def snapshot():
        return {"free": list(cache._free.keys()), "stats": cache.stats()}

    for _ in range(n_ops):
        r = rng.random()
        rec = {}
        try:
            if r < 0.25:
                d = docs[int(rng.integers(0, len(docs)))]
                n = int(rng.integers(1, len(d) + 1))
                toks = d[:n] + [int(t) for t in rng.integers(0, 6, int(rng.integers(0, 5)))]
                rec = {"op": "match", "tokens": toks}
                hit = cache.match_prefix(toks)
                rec["res"] = {"n_tokens": hit.n_tokens, "blocks": list(hit.block_ids),
                              "node": h_of(hit.node)}
                last_hit = {"blocks": list(hit.block_ids), "node": rec["res"]["node"],
                            "tokens": toks}
            elif r < 0.45:
                # publish a block-aligned chain: either the last hit's request
                # (prefix blocks reused, rest freshly allocated) or a new doc slice
                if last_hit["tokens"] and rng.random() < 0.6:
                    toks = last_hit["tokens"]
                    prefix_blocks = list(last_hit["blocks"])
                    parent = last_hit["node"] if rng.random() < 0.4 else None
                else:
                    d = docs[int(rng.integers(0, len(docs)))]
                    toks = d[:int(rng.integers(1, len(d) + 1))]
                    prefix_blocks, parent = [], None
                n_al = (len(toks) // bs) * bs
                toks = toks[:n_al]
                nb = n_al // bs - len(prefix_blocks)
                if parent is not None:
                    prefix_blocks = []
                    nb = n_al // bs
                if nb < 0 or n_al == 0:
                    continue
                rec = {"op": "insert", "tokens": toks, "nb": nb,
                       "prefix_blocks": prefix_blocks, "parent": parent}
                got = []
                try:
                    for _ in range(nb):
                        got.append(cache.alloc_block())
                except ref_radix.OutOfKVCacheError:
                    for b in got:
                        cache._free_block(b)
                    rec["alloc"] = got
                    raise
                rec["alloc"] = got
                node = cache.insert(toks, prefix_blocks + got,
                                    parent=handles[parent] if parent else None)
                rec["res"] = h_of(node)
            elif r < 0.57 and len(handles) > 1:
                hd = int(rng.integers(1, len(handles)))
                rec = {"op": "acquire", "node": hd}
                cache.acquire(handles[hd])
                pinned.append(hd)
            elif r < 0.70 and len(handles) > 1:
                if pinned and rng.random() < 0.9:
                    hd = pinned.pop(int(rng.integers(0, len(pinned))))
                else:
                    hd = int(rng.integers(1, len(handles)))
                rec = {"op": "release", "node": hd}
                cache.release(handles[hd])
            elif r < 0.80:
                rec = {"op": "evict", "n": int(rng.integers(1, 6))}
                rec["res"] = cache.evict(rec["n"])
            elif r < 0.88:
                rec = {"op": "ensure_free", "n": int(rng.integers(1, 16))}
                cache.ensure_free(rec["n"])
            elif r < 0.93:
                rec = {"op": "alloc"}
                rec["res"] = cache.alloc_block()
            else:
                rec = {"op": "free", "bid": int(rng.integers(0, 40))}
                cache._free_block(rec["bid"])
        except Exception as e:      # noqa: BLE001 - the error class is the result
            rec["error"] = type(e).__name__
        if rec:
            ops.append({**rec, "after": snapshot()})
    return {"n_blocks": 40, "block_size": bs, "ops": ops,
            "final_tree": tree_sig(cache._root)}


def tree_sig(n):
    return [list(n.tokens), list(n.blocks), n.refcnt,
            [[k, tree_sig(c)] for k, c in n.children.items()]]


def engine_meta(ref_radix, LLMEngine, seed=9):
    """Block-table growth + speculative rollback as the reference engine does it."""
    clock = itertools.count()
    ref_radix.time.monotonic = lambda: float(next(clock))
    bs = 16
    cache = ref_radix.RadixPagedKVCache(n_blocks=256, block_size=bs, n_layers=1,
                                        n_kv_heads=1, head_dim=1)

    class Stub:                      # the engine state _ensure_capacity touches
        kv = cache

        def _preempt_oldest(self):
            raise ref_radix.OutOfKVCacheError("preempt not modelled in fixture")

    class Seq:
        def __init__(self):
            self.block_table = []
            self.n_tokens = 0

    rng = np.random.default_rng(seed)
    seqs = [Seq() for _ in range(6)]
    trace = []
    for step in range(40):
        i = int(rng.integers(0, len(seqs)))
        s = seqs[i]
        gamma = int(rng.choice([1, 4, 8]))
        t = gamma + 1
        LLMEngine._ensure_capacity(Stub(), s, s.n_tokens + t)
        # observe where each written token lands, via unique markers
        marks = (np.arange(t, dtype=np.float32) + 1000.0 * (step + 1)).reshape(t, 1, 1)
        cache.write_layer(s.block_table, s.n_tokens, 0, marks, marks)
        flat = cache.k_pool[0, :, :, 0, 0].reshape(-1)
        slots = [int(np.flatnonzero(flat == m)[0]) for m in marks.reshape(-1)]
        start = s.n_tokens
        s.n_tokens += t
        rejected = int(rng.integers(0, gamma + 1))
        target = s.n_tokens - rejected
        if s.n_tokens > target:          # speculative.py:88-89
            s.n_tokens = target
        trace.append({"seq": i, "start": start, "t": t, "rejected": rejected,
                      "slots": slots, "table": list(s.block_table),
                      "n_tokens": s.n_tokens, "free": list(cache._free.keys())})
    return {"block_size": bs, "n_blocks": 256, "n_seqs": len(seqs), "trace": trace}


ROPE_CASES = [
    # name, table rows, head_dim, base, scaling_factor, original_max_pos, interleaved
    ("plain_hs", 8192, 128, 10000.0, 1.0, 4096, False),
    ("plain_il", 8192, 128, 10000.0, 1.0, 4096, True),
    ("llama3_hs", 8192, 128, 500000.0, 1.0, 4096, False),
    ("yarn_hs", 2048, 64, 10000.0, 4.0, 512, False),
    ("yarn_il", 2048, 64, 10000.0, 4.0, 512, True),
]


def rope_goldens(build_rope_cache, apply_rope, seed=21):
    """Per ROPE_CASES entry: the table rows the case uses, a digest of the
    whole cos / sin tables, seeded (T, H, D) inputs and apply_rope's output."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, rows, d, base, scale, omax, il in ROPE_CASES:
        cos, sin = build_rope_cache(rows, d, base, scaling_factor=scale,
                                    original_max_pos=omax, dtype=np.float32)
        x = rng.standard_normal((17, 3, d)).astype(np.float32)
        pos = rng.integers(0, rows, size=17).astype(np.int64)
        pos[:3] = [0, 1, rows - 1]
        out[name + "_table_digest"] = np.frombuffer(digest(cos, sin).encode(), dtype=np.uint8)
        out[name + "_cos_rows"], out[name + "_sin_rows"] = cos[pos], sin[pos]
        out[name + "_x"], out[name + "_pos"] = x, pos
        out[name + "_out"] = apply_rope(x, cos, sin, positions=pos, interleaved=il)
    return out


def model_goldens(ModelConfig, build_tiny_model, LLMEngine, SamplingParams,
                  SpeculativeDecoder):
    """Reference tiny models (vocab 264, hidden 64, intermediate 128, 2 layers,
    4 query / 2 KV heads, head_dim 16; draft = that config scaled by 0.5,
    seeds 42 and 99, block size 8, 64 blocks) and the prompt of the
    reference's conftest (10 tokens from default_rng(1))."""
    cfg = ModelConfig(vocab_size=264, hidden_size=64, intermediate_size=128,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2)
    target, tw = build_tiny_model(cfg, seed=42)
    dcfg = cfg.scaled(0.5)
    draft, dw = build_tiny_model(dcfg, seed=99)
    prompt = list(map(int, np.random.default_rng(1).integers(0, 256, 10)))

    def engine(m):
        return LLMEngine(m, None, block_size=8, n_blocks=64)

    out = {"prompt": np.asarray(prompt, dtype=np.int64)}
    for tag, c in (("t", cfg), ("d", dcfg)):
        out[f"{tag}.config"] = np.asarray(
            [c.vocab_size, c.hidden_size, c.intermediate_size, c.num_hidden_layers,
             c.num_attention_heads, c.num_key_value_heads, c.head_dim], dtype=np.int64)
        out[f"{tag}.rope"] = np.asarray([c.rope_theta, c.rms_norm_eps,
                                         c.max_position_embeddings], dtype=np.float64)
    for tag, w in (("t", tw), ("d", dw)):
        for k, v in w.items():
            out[f"{tag}.{k}"] = np.asarray(v, dtype=np.float32)
    e = engine(target)
    seq = e.create_sequence(prompt, SamplingParams(max_tokens=1))
    out["logits_full"] = e.prefill(seq).copy()
    e = engine(target)
    seq = e.create_sequence(prompt[:7], SamplingParams(max_tokens=1))
    e.prefill(seq)
    out["logits_incremental"] = e.forward_ids(seq, prompt[7:], allow_unconfirmed=True)
    e = engine(target)
    seq = e.create_sequence(prompt, SamplingParams(max_tokens=1))
    e.prefill(seq)
    seq.n_tokens = 5
    out["logits_rewrite"] = e.forward_ids(seq, prompt[5:], allow_unconfirmed=True)
    greedy = SamplingParams(max_tokens=16, temperature=0.0, seed=7)
    toks, _ = engine(target).generate(prompt, greedy)
    out["greedy_tokens"] = np.asarray(toks, dtype=np.int64)
    # teacher-forced logits over prompt + greedy tokens: the argmax margins
    e = engine(target)
    seq = e.create_sequence(prompt + toks, SamplingParams(max_tokens=1))
    seq.block_table = []
    seq.n_tokens = 0
    out["logits_teacher"] = e.forward_ids(seq, prompt + toks)
    for gamma in (1, 2, 4, 8):
        sd = SpeculativeDecoder(engine(target), engine(draft), num_speculative_tokens=gamma)
        o, _ = sd.generate(prompt, greedy)
        out[f"spec_tokens_{gamma}"] = np.asarray(o, dtype=np.int64)
        out[f"spec_stats_{gamma}"] = np.asarray([sd.stats.steps, sd.stats.drafted,
                                                sd.stats.accepted], dtype=np.int64)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to a Chenxing checkout")
    ap.add_argument("--only", choices=["rope", "model"], default=None)
    args = ap.parse_args()
    if args.only == "model" or args.only is None:
        sys.path.insert(0, args.reference)
        from chenxing.core.sampler import SamplingParams
        from chenxing.engine.engine import LLMEngine
        from chenxing.engine.speculative import SpeculativeDecoder
        from chenxing.model.config import ModelConfig
        from chenxing.model.transformer import build_tiny_model
        np.savez_compressed(os.path.join(HERE, "tiny_model.npz"),
                            **model_goldens(ModelConfig, build_tiny_model, LLMEngine,
                                            SamplingParams, SpeculativeDecoder))
        print("tiny_model.npz written to", HERE)
        if args.only == "model":
            return
    if args.only == "rope":
        sys.path.insert(0, args.reference)
        from chenxing.core.tensor import apply_rope, build_rope_cache
        np.savez_compressed(os.path.join(HERE, "rope.npz"),
                            **rope_goldens(build_rope_cache, apply_rope))
        print("rope.npz written to", HERE)
        return
    sys.path.insert(0, args.reference)
    sys.path.insert(0, ROOT)
    import ml_dtypes
    from chenxing.core import attention as ref_attn
    from chenxing.core.tensor import CausalMask
    from chenxing.engine import radix_kv as ref_radix
    from chenxing.engine.engine import LLMEngine

    bf16 = ml_dtypes.bfloat16
    sys.path.insert(0, HERE)
    arrs, cases = attention_outputs(ref_attn, CausalMask)
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **arrs)
    with open(os.path.join(HERE, "attention_cases.json"), "w") as f:
        json.dump(cases, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "paged_cfg1.npz"),
                        **paged_cfg1(ref_radix.RadixPagedKVCache, ref_attn.flash_attention,
                                     CausalMask))
    np.savez_compressed(os.path.join(HERE, "paged_bf16.npz"),
                        **paged_bf16(ref_radix.RadixPagedKVCache, ref_attn.flash_attention,
                                     CausalMask, bf16))
    with open(os.path.join(HERE, "radix_ops.json"), "w") as f:
        json.dump(radix_script(ref_radix), f)
    with open(os.path.join(HERE, "engine_meta.json"), "w") as f:
        json.dump(engine_meta(ref_radix, LLMEngine), f)
    from chenxing.core.tensor import apply_rope, build_rope_cache
    np.savez_compressed(os.path.join(HERE, "rope.npz"),
                        **rope_goldens(build_rope_cache, apply_rope))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
