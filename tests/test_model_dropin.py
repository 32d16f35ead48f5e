"""The reference's tiny model and speculative decoder, end to end, over the
KV path — the invariants of its tests/test_transformer.py:7-23 and
tests/test_speculative.py:14-21 with its own weights and goldens
(tests/golden/tiny_model.npz, written by running the reference).

* CPU: the restated model / engine (tests/tiny_model.py) over the oracle
  cache and oracle attention reproduces the reference's logits and tokens
  (pins the restatement).
* GPU: the same with ``chenxing_b200.RadixPagedKVCache`` (fp32 pool, every
  write_layer / read_layer a libcxkv kernel) and ``chenxing_b200.flash_attention``
  swapped in, as INTEGRATION.md's two-import swap does: logits within the
  reference's 1e-4, incremental == full prefill, rollback + rewrite
  idempotent, greedy tokens and speculative greedy output (gamma 1, 2, 4, 8)
  token for token equal to the reference's.
"""
import os

import numpy as np
import pytest

from tiny_model import TinyDecoder, TinyEngine, speculative_greedy

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny_model.npz")
LOGIT_ATOL = 1e-4        # the reference's own bar (tests/test_transformer.py:14,23)


def _run(make_cache, flash, CausalMask, gammas=(1, 2, 4, 8)):
    g = np.load(GOLDEN)
    prompt = [int(x) for x in g["prompt"]]
    tgt = TinyDecoder(g, "t", flash, CausalMask)
    dft = TinyDecoder(g, "d", flash, CausalMask)
    from tiny_model import TinySeq
    e = TinyEngine(tgt, make_cache)
    full = e.prefill(TinySeq(prompt), prompt)
    e = TinyEngine(tgt, make_cache)
    s = TinySeq(prompt[:7])
    e.prefill(s, prompt[:7])
    inc = e.forward_ids(s, prompt[7:])
    e = TinyEngine(tgt, make_cache)
    s = TinySeq(prompt)
    first = e.prefill(s, prompt)
    s.n_tokens = 5                                   # metadata-only rollback
    rew = e.forward_ids(s, prompt[5:])
    toks = TinyEngine(tgt, make_cache).generate_greedy(prompt, 16)
    spec = {gm: speculative_greedy(TinyEngine(tgt, make_cache), TinyEngine(dft, make_cache),
                                   prompt, gm, 16) for gm in gammas}
    return g, {"full": full, "inc": inc, "first": first, "rew": rew, "toks": toks, "spec": spec}


def _check(g, r):
    assert np.abs(r["full"] - g["logits_full"]).max() < LOGIT_ATOL
    assert np.abs(r["inc"] - g["logits_incremental"]).max() < LOGIT_ATOL
    assert np.abs(r["rew"] - g["logits_rewrite"]).max() < LOGIT_ATOL
    # the reference's own invariants, on this path
    assert np.abs(r["full"] - r["inc"][-1]).max() < LOGIT_ATOL
    assert np.abs(r["first"] - r["rew"][-1]).max() < LOGIT_ATOL
    assert r["toks"] == g["greedy_tokens"].tolist()
    for gm, (out, stats) in r["spec"].items():
        assert out == g[f"spec_tokens_{gm}"].tolist() == r["toks"], f"gamma {gm}"
        assert stats == g[f"spec_stats_{gm}"].tolist(), f"gamma {gm}"


def test_tiny_model_restatement_matches_reference_goldens():
    from oracle.attention import CausalMask, flash_attention
    from oracle.radix_kv import OraclePagedKVCache
    g, r = _run(lambda nb, bs, L, hk, hd: OraclePagedKVCache(nb, bs, L, hk, hd),
                flash_attention, CausalMask, gammas=(1, 8))
    _check(g, r)


@pytest.mark.gpu
def test_reference_model_runs_through_the_drop_ins():
    import chenxing_b200 as cx
    from chenxing_b200 import _lib
    _lib.device_flags(clear=True)
    g, r = _run(lambda nb, bs, L, hk, hd: cx.RadixPagedKVCache(nb, bs, L, hk, hd),
                cx.flash_attention, cx.CausalMask)
    _check(g, r)
    assert _lib.device_flags(clear=True) == 0
