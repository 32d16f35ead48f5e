"""Seeded paged-attention cases for the GPU parity tests (oracle = NumPy)."""
from __future__ import annotations

import numpy as np
import torch

from conftest import record_margin
from oracle.attention import CausalMask, flash_attention, naive_attention

BF16_RTOL = 2e-2     # bf16 pools: max|out - ref| <= 2e-2 * max|ref| per sequence
F32_ATOL = 1e-5      # fp32 pools: max|out - ref| <= 1e-5


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned as float32 (what the pool stores)."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16) \
        .float().numpy()


class PagedCase:
    """A cache with scattered block tables filled with seeded K/V, plus queries.

    ctx[b] counts every cached token of sequence b, including its q_lens[b]
    query tokens (already appended), as the model's forward does.
    """

    def __init__(self, *, hq, hk, d, ctx, q_lens=None, dtype="bfloat16", seed=0,
                 n_layers=1, layer=0, window=None, q_dtype=torch.float32, q_scale=1.0,
                 kv_scale=1.0, spare_blocks=7, bs=16):
        from chenxing_b200 import RadixPagedKVCache, slot_mapping
        rng = np.random.default_rng(seed)                 # K, V, Q values
        rng_place = np.random.default_rng(seed + 7777)    # physical placement
        self.hq, self.hk, self.d, self.layer, self.window = hq, hk, d, layer, window
        self.ctx = np.asarray(ctx, dtype=np.int64)
        self.verify = q_lens is not None
        self.q_lens = np.asarray(q_lens if q_lens is not None else [1] * len(ctx), dtype=np.int64)
        self.bs = bs
        nb_need = [max(1, -(-int(c) // bs)) for c in self.ctx]
        n_blocks = sum(nb_need) + spare_blocks
        self.cache = RadixPagedKVCache(n_blocks, bs, n_layers, hk, d, dtype=dtype,
                                       host_io=False)
        perm = rng_place.permutation(n_blocks)
        self.tables, o = [], 0
        for n in nb_need:
            self.tables.append([int(x) for x in perm[o:o + n]])
            o += n
        total = int(self.ctx.sum())
        k = (rng.standard_normal((total, hk, d)) * kv_scale).astype(np.float32)
        v = (rng.standard_normal((total, hk, d)) * kv_scale).astype(np.float32)
        slots = slot_mapping(self.tables, [0] * len(ctx), self.ctx, bs)
        if total:
            self.cache.append_batch(layer, k, v, slots)
        if dtype == "bfloat16":
            k, v = bf16_round(k), bf16_round(v)
        elif dtype == "float16":            # round-to-nearest-even, as the pool stores
            k = k.astype(np.float16).astype(np.float32)
            v = v.astype(np.float16).astype(np.float32)
        self.k, self.v = k, v
        self.q = (rng.standard_normal((int(self.q_lens.sum()), hq, d)) * q_scale).astype(np.float32)
        self.q_dev = torch.from_numpy(self.q).to(q_dtype).cuda()
        if q_dtype == torch.bfloat16:
            self.q = bf16_round(self.q)

    def batch(self, **kw):
        from chenxing_b200 import PagedBatch
        return PagedBatch(self.cache, self.tables, self.ctx, n_q_heads=self.hq,
                          q_lens=self.q_lens if self.verify else None, window=self.window, **kw)

    def run(self, batch=None, layer=None):
        batch = batch or self.batch()
        layer = self.layer if layer is None else layer
        fn = self.cache.verify_batch if self.verify else self.cache.decode_batch
        out = fn(layer, self.q_dev, batch)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    def oracle(self):
        outs, ko, qo = [], 0, 0
        for b in range(len(self.ctx)):
            c, ql = int(self.ctx[b]), int(self.q_lens[b])
            qb = self.q[qo:qo + ql]
            if c == 0:
                outs.append(np.zeros_like(qb))
            else:
                q4 = qb.transpose(1, 0, 2)[None]
                k4 = self.k[ko:ko + c].transpose(1, 0, 2)[None]
                v4 = self.v[ko:ko + c].transpose(1, 0, 2)[None]
                if self.window is None:
                    o = flash_attention(q4, k4, v4, CausalMask())
                else:
                    o = naive_attention(q4, k4, v4, CausalMask(self.window))
                outs.append(o[0].transpose(1, 0, 2))
            ko += c
            qo += ql
        return outs

    def check(self, out, atol=None, rtol=None):
        """Compare per sequence; returns the worst normalised error (error /
        bound), which the terminal summary also reports per test."""
        refs = self.oracle()
        worst, qo = 0.0, 0
        for b, ref in enumerate(refs):
            got = out[qo:qo + len(ref)]
            qo += len(ref)
            err = float(np.abs(got - ref).max()) if ref.size else 0.0
            assert np.isfinite(got).all(), f"non-finite output for sequence {b}"
            if atol is not None:
                assert err <= atol, f"seq {b} ctx {self.ctx[b]}: max abs err {err} > {atol}"
                worst = max(worst, err / atol)
            else:
                scale = float(np.abs(ref).max()) if ref.size else 0.0
                bound = rtol * scale
                assert err <= bound + 1e-30, \
                    f"seq {b} ctx {self.ctx[b]}: max abs err {err} > {rtol} * {scale}"
                worst = max(worst, err / bound if bound > 0 else 0.0)
        record_margin(worst)
        return worst


def pool_rows(cache, layer, table, lo, hi):
    """K, V of positions [lo, hi) of one sequence, read straight out of the
    pool tensors with torch indexing (checker side, not the product path);
    float32 NumPy arrays of shape (hi - lo, H, D)."""
    bs = cache.block_size
    pos = torch.arange(lo, hi, device=cache.device)
    bt = torch.as_tensor(table, dtype=torch.int64, device=cache.device)[pos // bs]
    k = cache._k[layer, bt, :, pos % bs]
    v = cache._v[layer, bt, :, pos % bs]
    return k.float().cpu().numpy(), v.float().cpu().numpy()


def oracle_rows(q, k, v, window=None):
    """Oracle attention of the last len(q) positions of a key run: q (T, hq, D),
    k / v (S, hk, D) float32 -> (T, hq, D).  With a window the run may start
    after position 0: the mask depends only on position differences."""
    q4 = np.ascontiguousarray(q.transpose(1, 0, 2)[None])
    k4 = np.ascontiguousarray(k.transpose(1, 0, 2)[None])
    v4 = np.ascontiguousarray(v.transpose(1, 0, 2)[None])
    if window is None:
        o = flash_attention(q4, k4, v4, CausalMask())
    else:
        o = naive_attention(q4, k4, v4, CausalMask(window))
    return o[0].transpose(1, 0, 2)


def assert_close_rows(got, ref, rtol=BF16_RTOL, what=""):
    assert np.isfinite(got).all(), f"non-finite output {what}"
    err = float(np.abs(got - ref).max())
    bound = rtol * float(np.abs(ref).max())
    assert err <= bound, f"{what}: max abs err {err} > {bound}"
    worst = err / bound if bound else 0.0
    record_margin(worst)
    return worst


def claim_blocks(index, ids):
    """Take ``ids`` out of an index's FIFO free list (harness placement of
    scattered tables); works on the product index and the oracle alike."""
    for b in ids:
        del index._free[int(b)]
