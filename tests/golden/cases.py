"""Seeded input definitions shared by make_golden.py and the tests.

Only outputs and a SHA-256 digest of these inputs are stored in the fixtures;
the tests rebuild the inputs here and first check the digest, so a change in
NumPy's random streams shows up as a digest mismatch, not as a parity failure.
"""
from __future__ import annotations

import hashlib

import numpy as np

try:                                    # bf16 pools of the reference use ml_dtypes
    import ml_dtypes
    BF16 = ml_dtypes.bfloat16
except ImportError:                     # pragma: no cover - present in this image
    BF16 = None


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def attention_cases():
    """List of dicts: name, q, k, v, mask ('none'|'causal'|'explicit'), window,
    explicit (bool array or None), use ('flash'|'naive'), scale."""
    cases = []

    def add(name, q, k, v, mask="none", window=None, explicit=None, use="flash",
            scale=None):
        cases.append(dict(name=name, q=q, k=k, v=v, mask=mask, window=window,
                          explicit=explicit, use=use, scale=scale))

    # the reference's tests/test_attention.py SHAPES (b, hq, sq, hk, d)
    for b, hq, sq, hk, d in [(1, 2, 5, 2, 8), (2, 4, 17, 4, 12), (1, 4, 64, 2, 8)]:
        rng = np.random.default_rng(b * 100 + sq)
        q = rng.standard_normal((b, hq, sq, d)).astype(np.float32)
        k = rng.standard_normal((b, hk, sq, d)).astype(np.float32)
        v = rng.standard_normal((b, hk, sq, d)).astype(np.float32)
        add(f"shape_{b}_{hq}_{sq}_{hk}_{d}", q, k, v)
        add(f"shape_{b}_{hq}_{sq}_{hk}_{d}_naive", q, k, v, use="naive")
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 9, 8)).astype(np.float32) for _ in range(3))
    add("causal_9", q, k, v, "causal")
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((1, 1, 12, 8)).astype(np.float32) for _ in range(3))
    add("window_12_w4", q, k, v, "causal", window=4)
    rng = np.random.default_rng(7)
    q, k, v = (rng.standard_normal((1, 2, 10, 8)).astype(np.float32) for _ in range(3))
    add("incr_full", q, k, v, "causal")
    add("incr_row9", np.ascontiguousarray(q[:, :, 9:10]), k, v, "causal")
    # decode / verify with GQA group 4 over several 64-key blocks
    rng = np.random.default_rng(21)
    q = rng.standard_normal((2, 8, 1, 64)).astype(np.float32)
    k = rng.standard_normal((2, 2, 300, 64)).astype(np.float32)
    v = rng.standard_normal((2, 2, 300, 64)).astype(np.float32)
    add("decode_gqa4_300", q, k, v, "causal")
    add("decode_gqa4_300_w32", q, k, v, "causal", window=32, use="naive")
    q5 = rng.standard_normal((2, 8, 5, 64)).astype(np.float32)
    add("verify5_gqa4_300", q5, k, v, "causal")
    add("verify5_gqa4_300_w64", q5, k, v, "causal", window=64, use="naive")
    add("verify5_scale", q5, k, v, "causal", scale=0.3)
    # dv != d, and an explicit boolean mask
    rng = np.random.default_rng(5)
    q = rng.standard_normal((1, 2, 6, 8)).astype(np.float32)
    k = rng.standard_normal((1, 2, 6, 8)).astype(np.float32)
    v = rng.standard_normal((1, 2, 6, 4)).astype(np.float32)
    add("dv4", q, k, v, "causal")
    msk = rng.random((6, 6)) < 0.6
    msk[:, 0] = True
    add("explicit_mask", q, k, v, "explicit", explicit=msk)
    # bf16 K/V (ml_dtypes, round-to-nearest-even), fp32 q, Llama-shaped heads
    rng = np.random.default_rng(33)
    q = (rng.standard_normal((1, 32, 1, 128)) / np.sqrt(128)).astype(np.float32)
    k = (rng.standard_normal((1, 8, 200, 128)) / np.sqrt(128)).astype(np.float32).astype(BF16)
    v = (rng.standard_normal((1, 8, 200, 128)) / np.sqrt(128)).astype(np.float32).astype(BF16)
    add("bf16_decode_200", q, k, v, "causal")
    q9 = (rng.standard_normal((1, 32, 9, 128)) / np.sqrt(128)).astype(np.float32)
    add("bf16_verify9_w64", q9, k, v, "causal", window=64, use="naive")
    return cases


def case_digest(c) -> str:
    parts = [c["q"], c["k"].view(np.uint16) if c["k"].dtype == BF16 else c["k"],
             c["v"].view(np.uint16) if c["v"].dtype == BF16 else c["v"]]
    if c["explicit"] is not None:
        parts.append(c["explicit"])
    return digest(*parts)


def paged_bf16_inputs():
    """cfg2-shaped bf16 pool case: per sequence fp32 K/V (rounded to bf16 on
    write) for ctx+1 tokens and one fp32 query row per head."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    from chenxing_b200.workloads import small_bf16
    wl = small_bf16(seed=1)
    rng = np.random.default_rng(101)
    ks, vs, qs = [], [], []
    for b in range(wl.batch):
        c = int(wl.ctx_lens[b]) + 1
        ks.append((rng.standard_normal((c, wl.n_kv_heads, wl.head_dim)) / np.sqrt(128)).astype(np.float32))
        vs.append((rng.standard_normal((c, wl.n_kv_heads, wl.head_dim)) / np.sqrt(128)).astype(np.float32))
        qs.append((rng.standard_normal((wl.n_q_heads, wl.head_dim)) / np.sqrt(128)).astype(np.float32))
    return wl, ks, vs, qs
