"""Attention drop-ins backed by libcxkv (chenxing/core/attention.py:30-148).

``flash_attention`` and ``naive_attention`` keep the reference signatures and
return float32 in the caller's array kind (NumPy in -> NumPy out, torch in ->
CUDA tensor out).  Both run an exact fp32 online softmax on the GPU, so they
agree with the reference's blocked kernel to float32 rounding (``block_q`` /
``block_k`` only shaped the reference's NumPy loop and are accepted for
signature compatibility).  Decode-shaped fp32 calls (one query token, causal
mask, a key count that is a multiple of 16, head_dim 64 or 128) run the paged
fp32 decode kernel over a pool view of the dense K / V (``_dense_decode``:
TMA-staged, split across all SMs); every other call runs
``cx_attention_dense`` (the tiled generic kernel).  Where the reference flash kernel
returns NaN — a query row whose leading 64-key block is entirely outside its
sliding window (attention.py:108,110) — this returns the defined value that
``naive_attention`` returns (attention.py:146).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from ._arrays import to_device, to_numpy
from .tensor import CausalMask

__all__ = ["flash_attention", "naive_attention", "gqa_expand"]


def _is_torch(x) -> bool:
    return isinstance(x, torch.Tensor)


def gqa_expand(kv, heads_kv: int, heads_q: int):
    """(b, hk, s, d) -> (b, hq, s, d); query head h uses KV head h // (hq/hk)
    (attention.py:30-40).  Runs on the GPU; returns the input's array kind."""
    if heads_kv == heads_q:
        return kv
    dev = _lib.require_cuda()
    t = to_device(kv, dev, float_only=False).repeat_interleave(heads_q // heads_kv, dim=1)
    return t if _is_torch(kv) else to_numpy(t)


_DENSE_META: dict = {}   # (device, rows, blocks, keys) -> (block tables, context lengths)


def _dense_decode(qt, kt, vt, b, hq, hk, sk, d, window, scale, dev):
    """One query token per sequence over dense fp32 K / V through
    ``cx_paged_decode``.  K (b, hk, sk, d) with sk a multiple of 16 is a pool
    of one layer, one KV head and b * hk * sk / 16 blocks of 16 tokens, laid
    out [block][16][d]: (sequence, KV head) pair i owns blocks i * sk / 16 ..,
    in order.  Q (b, hq, 1, d) is then (b * hk) sequences of hq / hk query
    heads, and the output (b, hq, 1, d) the same rows.  The plan / split
    workspace comes from torch's allocator."""
    nb = sk // 16
    seqs = b * hk
    key = (dev, seqs, nb, sk)
    meta = _DENSE_META.get(key)
    if meta is None:
        tables = torch.arange(seqs * nb, dtype=torch.int32, device=dev).view(seqs, nb)
        ctx = torch.full((seqs,), sk, dtype=torch.int32, device=dev)
        meta = _DENSE_META[key] = (tables, ctx)
        if len(_DENSE_META) > 64:
            _DENSE_META.pop(next(iter(_DENSE_META)))
    tables, ctx = meta
    pool = _lib.CxPool(kt.data_ptr(), vt.data_ptr(), 1, seqs * nb, 16, 1, d, _lib.CX_F32, 0)
    batch = _lib.CxAttnBatch(tables.data_ptr(), nb, ctx.data_ptr(), None, seqs, 1, hq // hk,
                             scale, 0, window)
    lib = _lib.lib()
    need = int(lib.cx_paged_workspace_bytes(pool, batch))
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
    out = torch.empty((b, hq, 1, d), dtype=torch.float32, device=dev)
    _lib.check(lib.cx_paged_decode(pool, 0, batch, qt.data_ptr(), _lib.cx_dtype(qt.dtype),
                                   out.data_ptr(), ws.data_ptr(), need, 1, _lib.stream_ptr(dev)),
               "flash_attention (paged decode view)")
    return out


def _attention(q, k, v, mask, scale, name: str):
    dev = _lib.require_cuda(q.device if _is_torch(q) and q.is_cuda else None)
    b, hq, sq, d = (int(x) for x in q.shape)
    hk, sk = int(k.shape[1]), int(k.shape[2])
    dv = int(v.shape[-1])
    if hq % hk != 0:
        raise ValueError(f"GQA requires hq % hk == 0, got hq={hq}, hk={hk}")
    scale = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    mask_kind, window, mask_t = 0, 0, None
    if isinstance(mask, CausalMask) or type(mask).__name__ == "CausalMask":
        mask_kind = 1
        sw = getattr(mask, "sliding_window", None)
        window = int(sw) if sw is not None else 0
        if sw is not None and window <= 0:
            # w <= 0 attends nothing (j + w > pos never holds for j <= pos)
            mask_kind, mask_t = 2, torch.zeros((sq, sk), dtype=torch.uint8, device=dev)
    elif mask is not None:
        m = mask if _is_torch(mask) else np.asarray(mask, dtype=bool)
        if tuple(m.shape) != (sq, sk):
            raise ValueError(f"mask shape {tuple(m.shape)} != ({sq}, {sk})")
        mask_kind = 2
        mask_t = (m.to(dev, torch.uint8) if _is_torch(m)
                  else torch.from_numpy(np.ascontiguousarray(m, dtype=np.uint8)).to(dev))
    qt = to_device(q, dev)
    kt = to_device(k, dev)
    vt = to_device(v, dev)
    if kt.dtype != vt.dtype:
        vt = vt.to(kt.dtype)
    if (mask_kind == 1 and sq == 1 and sk > 0 and sk % 16 == 0 and d == dv and d in (64, 128)
            and kt.dtype == torch.float32 and qt.dtype in (torch.float32, torch.bfloat16)
            and hq // hk <= 64 and b * hk < (1 << 24)):
        out = _dense_decode(qt, kt, vt, b, hq, hk, sk, d, window, scale, dev)
        return out if _is_torch(q) else to_numpy(out)
    out = torch.empty((b, hq, sq, dv), dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().cx_attention_dense(
        qt.data_ptr(), _lib.cx_dtype(qt.dtype), kt.data_ptr(), vt.data_ptr(),
        _lib.cx_dtype(kt.dtype), b, hq, sq, hk, sk, d, dv, mask_kind, window,
        _lib.ptr(mask_t), scale, out.data_ptr(), _lib.stream_ptr(dev)), name)
    return out if _is_torch(q) else to_numpy(out)


def flash_attention(q, k, v, mask=None, scale=None, *, block_q: int = 64, block_k: int = 64):
    """Online-softmax attention; q (b, hq, sq, d), k (b, hk, sk, d),
    v (b, hk, sk, dv) -> float32 (b, hq, sq, dv) (attention.py:43-116)."""
    return _attention(q, k, v, mask, scale, "flash_attention")


def naive_attention(q, k, v, mask=None, scale=None):
    """Same contract as flash_attention; fully masked rows give 0
    (attention.py:119-148)."""
    return _attention(q, k, v, mask, scale, "naive_attention")
