"""Batched paged attention over a RadixPagedKVCache.

The reference decodes one sequence at a time (chenxing/engine/scheduler.py:59-74,
chenxing/engine/engine.py:110-129): per layer ``write_layer`` then
``read_layer`` + ``flash_attention``.  ``PagedBatch`` carries the same
per-sequence metadata (block tables, context lengths, query lengths) for a
whole batch as device arrays, so one ``cx_kv_append`` and one
``cx_paged_decode`` / ``cx_paged_verify`` launch serve every sequence of a
layer.  Tables and lengths are exactly the reference's ``Sequence.block_table``
and ``n_tokens`` values; nothing here changes them.
"""
from __future__ import annotations

import itertools
import math

import numpy as np
import torch

from . import _lib
from ._arrays import to_device, upload

__all__ = ["PagedBatch", "slot_mapping", "decode_batch", "verify_batch"]


def slot_mapping(block_tables, starts, counts, block_size: int) -> np.ndarray:
    """Physical slots for positions [starts[b], starts[b] + counts[b]) of each
    sequence, concatenated: ``table[p // bs] * bs + p % bs`` (the placement
    rule of write_layer, chenxing/engine/radix_kv.py:123-128)."""
    starts = np.asarray(starts, dtype=np.int64).reshape(-1)
    counts = np.asarray(counts, dtype=np.int64).reshape(-1)
    bs = int(block_size)
    # only the table entries each write range touches, gathered in one pass
    parts, lens = [], []
    for bt, s, c in zip(block_tables, starts.tolist(), counts.tolist()):
        if c == 0:
            lens.append(0)
            continue
        if len(bt) * bs < s + c:
            raise ValueError("block_table too short for requested write range")
        seg = bt[s // bs:(s + c - 1) // bs + 1]
        parts.append(seg)
        lens.append(len(seg))
    total = int(counts.sum())
    if total == 0:
        return np.zeros(0, dtype=np.int64)
    ids = np.fromiter(itertools.chain.from_iterable(parts), dtype=np.int64, count=sum(lens))
    seg_off = np.zeros(len(lens), dtype=np.int64)
    np.cumsum(lens[:-1], out=seg_off[1:])
    row_off = np.zeros(len(counts), dtype=np.int64)
    np.cumsum(counts[:-1], out=row_off[1:])
    pos = np.arange(total, dtype=np.int64) + np.repeat(starts - row_off, counts)
    base = np.repeat(seg_off - starts // bs, counts)        # table index -> ids index
    return ids[base + pos // bs] * bs + pos % bs


class PagedBatch:
    """Device metadata + workspace for batched decode / verify on one cache.

    block_tables: list of per-sequence block-id lists; ctx_lens: cached tokens
    per sequence INCLUDING the query tokens being attended (they are appended
    first, as in transformer.py:87-88); q_lens: query tokens per sequence
    (None = decode, one each); window: sliding window or None.
    """

    def __init__(self, cache, block_tables, ctx_lens, *, n_q_heads: int, q_lens=None,
                 window: int | None = None, scale: float | None = None,
                 table_stride: int | None = None) -> None:
        self.cache = cache
        self.device = cache.device
        self.n_q_heads = int(n_q_heads)
        if self.n_q_heads % cache.n_kv_heads:
            raise ValueError(f"GQA requires hq % hk == 0, got hq={n_q_heads}, hk={cache.n_kv_heads}")
        self.window = int(window) if window is not None else 0
        if window is not None and self.window <= 0:
            raise ValueError("window must be positive (or None)")
        self.scale = (1.0 / math.sqrt(cache.head_dim)) if scale is None else float(scale)
        self.verify = q_lens is not None
        self.table_stride = table_stride
        self._ws = None
        self._ws_bytes = 0
        self.set(block_tables, ctx_lens, q_lens)

    # ------------------------------------------------------------------ #
    def set(self, block_tables, ctx_lens, q_lens=None) -> None:
        """(Re)load tables and lengths; the next attention call re-plans."""
        bs = self.cache.block_size
        B = len(block_tables)
        ctx = np.asarray(ctx_lens, dtype=np.int64).reshape(-1)
        if ctx.shape[0] != B:
            raise ValueError("ctx_lens and block_tables differ in length")
        lens = np.fromiter(map(len, block_tables), dtype=np.int64, count=B)
        longest = int(lens.max(initial=0))
        stride = max(self.table_stride or 0, longest, 1)
        if self.table_stride is not None and longest > self.table_stride:
            raise ValueError("a block table is longer than table_stride")
        if np.any(ctx < 0) or np.any(ctx > lens * bs):
            raise ValueError("context length outside [0, len(block_table) * block_size]")
        ids = np.fromiter(itertools.chain.from_iterable(block_tables), dtype=np.int64,
                          count=int(lens.sum()))
        if ids.size and (ids.min() < 0 or ids.max() >= self.cache.n_blocks):
            raise IndexError(f"block id outside [0, {self.cache.n_blocks})")
        tab = np.zeros((B, stride), dtype=np.int32)
        tab[np.arange(stride) < lens[:, None]] = ids   # row-major mask order = concatenation
        self.batch = B
        self.stride = stride
        self.tables_host = [list(t) for t in block_tables]
        self.ctx_host = ctx
        self.block_tables = upload(tab, self.device)
        self.ctx_lens = upload(ctx.astype(np.int32), self.device)
        if self.verify:
            ql = np.asarray(q_lens, dtype=np.int64).reshape(-1)
            if ql.shape[0] != B or np.any(ql < 0) or np.any(ql > ctx):
                raise ValueError("q_lens must be per sequence and <= ctx_lens")
            qs = np.zeros(B + 1, dtype=np.int64)
            np.cumsum(ql, out=qs[1:])
            self.q_lens_host = ql
            self.q_start = upload(qs.astype(np.int32), self.device)
            self.max_q = int(ql.max(initial=1))
            self.total_q = int(qs[-1])
        else:
            self.q_lens_host = np.ones(B, dtype=np.int64)
            self.q_start = None
            self.max_q = 1
            self.total_q = B
        self._c = _lib.CxAttnBatch(self.block_tables.data_ptr(), self.stride,
                                   self.ctx_lens.data_ptr(),
                                   _lib.ptr(self.q_start), B, self.max_q, self.n_q_heads,
                                   self.scale, 0, self.window)
        need = int(_lib.lib().cx_paged_workspace_bytes(self.cache.cx_pool(), self._c))
        if need > self._ws_bytes:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
            self._ws_bytes = need
        self.needs_plan = True

    def advance(self, n: int = 1) -> None:
        """Every context grows by ``n`` tokens (one decode step); re-plans."""
        self.set(self.tables_host, self.ctx_host + n,
                 self.q_lens_host if self.verify else None)

    @property
    def kv_tokens(self) -> int:
        """Keys attended per layer (KV token-layers of one step and layer)."""
        if self.window:
            lo = np.maximum(0, self.ctx_host - self.q_lens_host - self.window + 1)
            return int(np.sum(self.ctx_host - lo))
        return int(self.ctx_host.sum())

    def kernel_kind(self, q_dtype=torch.bfloat16) -> str:
        """Which libcxkv kernel attends this batch: "generic", "mma" or "tcgen05"."""
        k = _lib.lib().cx_paged_kernel_kind(self.cache.cx_pool(), self._c,
                                            _lib.cx_dtype(q_dtype), int(self.verify))
        return _lib.KERNEL_KINDS[k]

    def c_struct(self) -> _lib.CxAttnBatch:
        return self._c

    @property
    def workspace(self) -> torch.Tensor:
        return self._ws


def _attend(cache, layer: int, q, batch: PagedBatch, out, replan, fn_name: str):
    if batch.cache is not cache:
        raise ValueError("PagedBatch belongs to a different cache")
    qt = to_device(q, cache.device)
    expect = (batch.total_q, batch.n_q_heads, cache.head_dim)
    if tuple(qt.shape) != expect:
        raise ValueError(f"q must have shape {expect}, got {tuple(qt.shape)}")
    if out is None:
        out = torch.empty(expect, dtype=torch.float32, device=cache.device)
    elif tuple(out.shape) != expect or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous float32 tensor of shape {expect}")
    do_plan = batch.needs_plan if replan is None else bool(replan)
    fn = getattr(_lib.lib(), fn_name)
    _lib.check(fn(cache.cx_pool(), int(layer), batch.c_struct(), qt.data_ptr(),
                  _lib.cx_dtype(qt.dtype), out.data_ptr(), batch.workspace.data_ptr(),
                  batch.workspace.numel(), int(do_plan), _lib.stream_ptr(cache.device)), fn_name)
    if do_plan:
        batch.needs_plan = False
    return out


def decode_batch(cache, layer: int, q, batch: PagedBatch, out=None, replan=None):
    """One query token per sequence: q (B, hq, D) -> float32 (B, hq, D)."""
    if batch.verify:
        raise ValueError("decode_batch needs a PagedBatch built without q_lens")
    return _attend(cache, layer, q, batch, out, replan, "cx_paged_decode")


def verify_batch(cache, layer: int, q, batch: PagedBatch, out=None, replan=None):
    """q_lens[b] query tokens per sequence (speculative verify / prefill chunk):
    q (sum q_lens, hq, D) -> float32 (sum q_lens, hq, D)."""
    if not batch.verify:
        raise ValueError("verify_batch needs a PagedBatch built with q_lens")
    return _attend(cache, layer, q, batch, out, replan, "cx_paged_verify")
