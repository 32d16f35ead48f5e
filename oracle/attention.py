"""Attention oracle (NumPy) — TEST INFRASTRUCTURE ONLY, never the product path.

Restates the reference's attention kernels:

* ``gqa_expand``       — ``chenxing/core/attention.py:30-40``
* ``attend_map``       — mask construction of ``chenxing/core/attention.py:75-86``
                         and ``naive_attention`` ``:134-141`` for
                         ``CausalMask(sliding_window)`` (``chenxing/core/tensor.py:183-186``)
* ``flash_attention``  — blocked online softmax, ``chenxing/core/attention.py:43-116``
* ``naive_attention``  — full softmax with masked rows mapped to zero,
                         ``chenxing/core/attention.py:119-148``

All arithmetic is float32 like the reference (inputs are up-cast with
``astype(np.float32)``; bf16 inputs are ``ml_dtypes.bfloat16`` arrays).
The reference flash kernel yields NaN for a query row whose first key block
is entirely masked by a sliding window (``exp(-inf - -inf)`` at
``attention.py:108,110``); this restatement reproduces that on purpose, and the
parity tests use ``naive_attention`` for every windowed case.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = ["CausalMask", "gqa_expand", "attend_map", "flash_attention",
           "naive_attention"]


@dataclass(frozen=True)
class CausalMask:
    """Causal mask marker with optional sliding window (core/tensor.py:183-186)."""
    sliding_window: int | None = None


def gqa_expand(kv: np.ndarray, heads_kv: int, heads_q: int) -> np.ndarray:
    """Query head ``h`` reads KV head ``h // (heads_q // heads_kv)`` (attention.py:30-40)."""
    if heads_kv == heads_q:
        return kv
    return np.repeat(kv, heads_q // heads_kv, axis=1)


def attend_map(sq: int, sk: int, sliding_window: int | None) -> np.ndarray:
    """Boolean (sq, sk) map, True = attend (attention.py:75-80).

    Query row ``i`` sits at absolute position ``i + sk - sq`` (incremental
    decode offset); it sees key ``j`` iff ``j <= pos`` and, with a window
    ``w``, ``j + w > pos``.
    """
    pos = np.arange(sq)[:, None] + (sk - sq)
    keys = np.arange(sk)[None, :]
    ok = keys <= pos
    if sliding_window is not None:
        ok = ok & (keys + sliding_window > pos)
    return ok


def _mask_to_map(mask, sq: int, sk: int) -> np.ndarray | None:
    if isinstance(mask, CausalMask) or type(mask).__name__ == "CausalMask":
        return attend_map(sq, sk, mask.sliding_window)
    if mask is None:
        return None
    m = np.asarray(mask, dtype=bool)
    if m.shape != (sq, sk):
        raise ValueError(f"mask shape {m.shape} != ({sq}, {sk})")
    return m


def flash_attention(q, k, v, mask=None, scale=None, *, block_q: int = 64,
                    block_k: int = 64) -> np.ndarray:
    """Blocked online-softmax attention; float32 output (attention.py:43-116).

    q (b, hq, sq, d); k (b, hk, sk, d); v (b, hk, sk, dv).  Running max ``mx``,
    running denominator ``den`` and rescaled accumulator ``num`` per query row,
    updated once per ``block_k`` keys; final divide by ``max(den, 1e-38)``.
    """
    b, hq, sq, d = q.shape
    hk, sk = k.shape[1], k.shape[2]
    dv = v.shape[-1]
    if hq % hk != 0:
        raise ValueError(f"GQA requires hq % hk == 0, got hq={hq}, hk={hk}")
    k = gqa_expand(k, hk, hq)
    v = gqa_expand(v, hk, hq)
    scale = float(1.0 / np.sqrt(d)) if scale is None else scale
    amap = _mask_to_map(mask, sq, sk)
    out = np.empty((b, hq, sq, dv), dtype=np.float32)
    for r0 in range(0, sq, block_q):
        r1 = min(r0 + block_q, sq)
        qt = q[:, :, r0:r1, :].astype(np.float32)
        mx = np.full((b, hq, r1 - r0, 1), -np.inf, dtype=np.float32)
        den = np.zeros((b, hq, r1 - r0, 1), dtype=np.float32)
        num = np.zeros((b, hq, r1 - r0, dv), dtype=np.float32)
        for c0 in range(0, sk, block_k):
            c1 = min(c0 + block_k, sk)
            s = np.einsum("bhid,bhjd->bhij", qt, k[:, :, c0:c1, :].astype(np.float32)) * scale
            if amap is not None:
                s = np.where(amap[None, None, r0:r1, c0:c1], s, -np.inf)
            mx_new = np.maximum(mx, s.max(axis=-1, keepdims=True))
            p = np.exp(s - mx_new)
            corr = np.exp(mx - mx_new)
            num = num * corr + np.einsum("bhij,bhjd->bhid", p,
                                         v[:, :, c0:c1, :].astype(np.float32))
            den = den * corr + p.sum(axis=-1, keepdims=True)
            mx = mx_new
        out[:, :, r0:r1, :] = num / np.maximum(den, 1e-38)
    return out


def naive_attention(q, k, v, mask=None, scale=None) -> np.ndarray:
    """Full-softmax attention, fully masked rows -> 0 (attention.py:119-148)."""
    b, hq, sq, d = q.shape
    hk, sk = k.shape[1], k.shape[2]
    k = gqa_expand(k, hk, hq)
    v = gqa_expand(v, hk, hq)
    scale = float(1.0 / np.sqrt(d)) if scale is None else scale
    s = np.einsum("bhid,bhjd->bhij", q.astype(np.float32), k.astype(np.float32)) * scale
    amap = _mask_to_map(mask, sq, sk)
    if amap is not None:
        s = np.where(amap[None, None], s, -np.inf)
    with np.errstate(invalid="ignore"):
        w = np.exp(s - s.max(axis=-1, keepdims=True))
    w = np.nan_to_num(w, nan=0.0, posinf=0.0, neginf=0.0)
    w = w / np.maximum(w.sum(axis=-1, keepdims=True), 1e-38)
    return np.einsum("bhij,bhjd->bhid", w, v.astype(np.float32))
