"""Seeded synthetic workloads for the KV hot path (host-side metadata + data).

The reference publishes no dataset for this path; every workload is synthetic
and seeded with ``numpy.random.default_rng(seed)``.  Shapes follow the five
configurations the benchmark and the parity tests use:

cfg1  8 seqs, ctx ~ U[64, 512], bs 16, Hq 8 / Hkv 2, D 64, fp32, tables are
      slices of a permutation of a 512-block pool, 32 decode steps.
cfg2  Llama-3-8B-shaped decode: B 64, ctx ~ U[1024, 8192], 32 layers,
      Hq 32 / Hkv 8, D 128, bf16 pool, Q/K/V ~ N(0, 1) / sqrt(128).
cfg3  radix prefix sharing: 256 requests in 4 groups sharing a prefix whose
      last block is partially filled (forces copy-on-write), Hkv 32, D 128.
cfg4  speculative verify: B 128, ctx ~ U[2048, 16384], gamma in {4, 8},
      window 4096, Hq 32 / Hkv 8, D 128, bf16.
cfg5  continuous-batching churn: lognormal ctx (median 2048, sigma 1.0,
      capped at 32768), Hkv 8, D 128, bf16, sharded by sequence.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

__all__ = ["DecodeWorkload", "cfg1", "cfg2_meta", "small_bf16", "verify_meta",
           "lognormal_ctx", "prefix_share_meta"]


@dataclass
class DecodeWorkload:
    """Block tables + context lengths for a batch of decode sequences."""
    n_layers: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    block_size: int
    n_blocks: int
    ctx_lens: np.ndarray                 # (B,) int64, tokens already cached
    block_tables: list                   # list[list[int]], capacity ctx+steps
    steps: int = 1
    dtype: str = "float32"
    extra: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return len(self.ctx_lens)


def _tables_from_perm(ctx_plus, block_size, perm):
    tables, o = [], 0
    for c in ctx_plus:
        nb = -(-int(c) // block_size)
        tables.append([int(x) for x in perm[o:o + nb]])
        o += nb
    if o > len(perm):
        raise ValueError("pool too small for the requested contexts")
    return tables


def cfg1(seed: int = 0, steps: int = 32):
    """cfg1 metadata and all float32 inputs (prefill K/V and per-step q/k/v).

    Returns (workload, data) where data holds ``k_pre``/``v_pre`` lists of
    (ctx_b, 2, 64) arrays and ``q``/``k``/``v`` of shape (steps, 8, H, 64).
    """
    rng = np.random.default_rng(seed)
    B, hq, hk, d, bs, nb = 8, 8, 2, 64, 16, 512
    ctx = rng.integers(64, 513, size=B).astype(np.int64)
    perm = rng.permutation(nb)
    tables = _tables_from_perm(ctx + steps, bs, perm)
    k_pre = [rng.standard_normal((int(c), hk, d)).astype(np.float32) for c in ctx]
    v_pre = [rng.standard_normal((int(c), hk, d)).astype(np.float32) for c in ctx]
    q = rng.standard_normal((steps, B, hq, d)).astype(np.float32)
    k = rng.standard_normal((steps, B, hk, d)).astype(np.float32)
    v = rng.standard_normal((steps, B, hk, d)).astype(np.float32)
    wl = DecodeWorkload(1, hq, hk, d, bs, nb, ctx, tables, steps, "float32")
    return wl, {"k_pre": k_pre, "v_pre": v_pre, "q": q, "k": k, "v": v}


def cfg2_meta(n_blocks: int, seed: int = 0, batch: int = 64, steps: int = 1,
              ctx_lo: int = 1024, ctx_hi: int = 8192, n_layers: int = 32,
              world: int = 1, rank: int = 0):
    """cfg2 metadata: tables scattered over an ``n_blocks`` pool by permutation.

    With ``world`` > 1 the contexts of a global batch of ``batch * world``
    sequences are drawn once and dealt to the ranks by length
    (``deal_by_context``: ``batch`` sequences each, near-equal KV tokens), and
    this returns rank ``rank``'s share; ``world`` = 1 is the plain batch."""
    from .sharding import deal_by_context
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch * world).astype(np.int64)
    if world > 1:
        ctx = ctx[deal_by_context(ctx, world)[rank]]
    perm = rng.permutation(n_blocks)
    tables = _tables_from_perm(ctx + steps, 16, perm)
    return DecodeWorkload(n_layers, 32, 8, 128, 16, n_blocks, ctx, tables, steps,
                          "bfloat16")


def small_bf16(seed: int = 0, batch: int = 6, ctx_lo: int = 17, ctx_hi: int = 700,
               n_blocks: int = 512, hq: int = 32, hk: int = 8, d: int = 128,
               bs: int = 16, steps: int = 1):
    """A cfg2-shaped case small enough for the NumPy oracle."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch).astype(np.int64)
    perm = rng.permutation(n_blocks)
    tables = _tables_from_perm(ctx + steps, bs, perm)
    return DecodeWorkload(1, hq, hk, d, bs, n_blocks, ctx, tables, steps, "bfloat16")


def verify_meta(n_blocks: int, seed: int = 0, batch: int = 128, gamma: int = 4,
                ctx_lo: int = 2048, ctx_hi: int = 16384, window: int = 4096,
                n_layers: int = 1):
    """cfg4 metadata: ctx counts cached tokens BEFORE the gamma+1 verify tokens."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch).astype(np.int64)
    perm = rng.permutation(n_blocks)
    tables = _tables_from_perm(ctx + gamma + 1, 16, perm)
    rejected = rng.integers(0, gamma + 1, size=batch).astype(np.int64)
    return DecodeWorkload(n_layers, 32, 8, 128, 16, n_blocks, ctx, tables, 1,
                          "bfloat16", {"gamma": gamma, "window": window,
                                       "rejected": rejected})


def lognormal_ctx(n: int, seed: int = 0, median: float = 2048.0, sigma: float = 1.0,
                  cap: int = 32768, lo: int = 16):
    """cfg5 context lengths: lognormal(mu=ln(median), sigma), clipped to [lo, cap]."""
    rng = np.random.default_rng(seed)
    c = rng.lognormal(mean=np.log(median), sigma=sigma, size=n)
    return np.clip(np.round(c), lo, cap).astype(np.int64)


def prefix_share_meta(seed: int = 0, n_groups: int = 4, per_group: int = 64,
                      prefix_tokens: int = 2048, block_size: int = 16,
                      suffix_lo: int = 128, suffix_hi: int = 512):
    """cfg3 shapes: per group a shared prefix of ``prefix_tokens + r_g`` tokens
    (r_g in [1, bs-1], so its last block is shared and partially filled) and a
    unique suffix length per request."""
    rng = np.random.default_rng(seed)
    tail = rng.integers(1, block_size, size=n_groups).astype(np.int64)
    suffix = rng.integers(suffix_lo, suffix_hi + 1,
                          size=(n_groups, per_group)).astype(np.int64)
    return {"prefix_tokens": prefix_tokens, "tail": tail, "suffix": suffix,
            "block_size": block_size}
