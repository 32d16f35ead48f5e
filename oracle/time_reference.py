"""Times the reference's own CPU path beside this repository's restatement of
it (oracle/), on the same sample and the same single core — TEST / BENCH
INFRASTRUCTURE, run where a checkout of the reference exists:

    python oracle/time_reference.py --reference <path-to-chenxing-checkout>

Sample: 4 sequences of the cfg2 decode workload (bf16 pool through
ml_dtypes, Hq 32 / Hkv 8, D 128), one layer, per sequence and decode step
write_layer -> read_layer -> flash_attention(CausalMask()) exactly as
chenxing/model/transformer.py:87-94 calls them.  Prints one JSON line with
both rates (KV token-layers/s) and their ratio; the GPU box has no reference
checkout, so bench.py's CPU arms time the restatement and this script shows
how closely it tracks the reference.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HQ, HK, D, BS = 32, 8, 128, 16


def _rate(cache_cls, attend, ctxs, seconds, bf16):
    rng = np.random.default_rng(0)
    need = sum(-(-(int(c) + 64) // BS) for c in ctxs)
    cache = cache_cls(need, BS, 1, HK, D, dtype=bf16)
    tables, o = [], 0
    for c in ctxs:
        n = -(-(int(c) + 64) // BS)
        tables.append(list(range(o, o + n)))
        o += n
    for c, t in zip(ctxs, tables):
        kv = (rng.standard_normal((int(c), HK, D)) / math.sqrt(D)).astype(np.float32)
        cache.write_layer(t, 0, 0, kv, kv)
    ctx = [int(c) for c in ctxs]
    units, steps = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for i, t in enumerate(tables):
            q = (rng.standard_normal((1, HQ, D)) / math.sqrt(D)).astype(np.float32)
            kn = (rng.standard_normal((1, HK, D)) / math.sqrt(D)).astype(np.float32)
            if ctx[i] + 1 > len(t) * BS:
                ctx[i] -= 32
            attend(cache, t, ctx[i], q, kn)
            ctx[i] += 1
            units += ctx[i]
        steps += 1
    return units / (time.perf_counter() - t0), steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--seconds", type=float, default=12.0)
    args = ap.parse_args()
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    sys.path.insert(0, args.reference)
    sys.path.insert(0, ROOT)
    import ml_dtypes
    from chenxing.core.attention import flash_attention as ref_flash
    from chenxing.core.tensor import CausalMask as RefMask
    from chenxing.engine.radix_kv import RadixPagedKVCache as RefCache
    from oracle.paged import attend_sequence
    from oracle.radix_kv import OraclePagedKVCache

    def ref_attend(cache, t, n_past, q, kn):
        cache.write_layer(t, n_past, 0, kn, kn)
        k_all, v_all = cache.read_layer(t, n_past + 1, 0)
        q4 = np.ascontiguousarray(np.transpose(q, (1, 0, 2))[None])
        k4 = np.ascontiguousarray(np.transpose(k_all, (1, 0, 2))[None])
        v4 = np.ascontiguousarray(np.transpose(v_all, (1, 0, 2))[None])
        return ref_flash(q4, k4, v4, RefMask())

    def port_attend(cache, t, n_past, q, kn):
        return attend_sequence(cache, t, n_past, 0, q, kn, kn)

    from chenxing_b200.workloads import cfg2_meta
    ctxs = [int(c) for c in cfg2_meta(n_blocks=64 * 600, seed=0).ctx_lens[:4]]
    bf16 = ml_dtypes.bfloat16
    ref, rs = _rate(RefCache, ref_attend, ctxs, args.seconds, bf16)
    port, ps = _rate(OraclePagedKVCache, port_attend, ctxs, args.seconds, bf16)
    print(json.dumps({"sample": f"4 cfg2 sequences (ctx {ctxs}), 1 layer, bf16 pool, 1 core",
                      "reference_kv_token_layers_per_s": ref, "reference_steps": rs,
                      "port_kv_token_layers_per_s": port, "port_steps": ps,
                      "port_over_reference": port / ref}))


if __name__ == "__main__":
    main()
