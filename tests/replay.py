"""Replay helpers for the golden metadata fixtures (shared by oracle and product tests)."""
from __future__ import annotations

import json
import os

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_json(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def tree_sig(node):
    return [list(node.tokens), list(node.blocks), node.refcnt,
            [[k, tree_sig(c)] for k, c in node.children.items()]]


def replay_radix(cache, fixture, oom_error):
    """Replay ``radix_ops.json`` on ``cache``; return a list of mismatch strings.

    ``cache`` must offer the reference API (alloc_block, _free_block,
    match_prefix, insert, acquire, release, evict, ensure_free, stats) and a
    ``_free`` mapping whose key order is the FIFO free-list order.
    """
    handles = [None]
    bad = []

    def h_of(node):
        for i, n in enumerate(handles):
            if n is node:
                return i
        handles.append(node)
        return len(handles) - 1

    for i, op in enumerate(fixture["ops"]):
        kind = op["op"]
        got = {}
        try:
            if kind == "match":
                hit = cache.match_prefix(op["tokens"])
                got["res"] = {"n_tokens": hit.n_tokens, "blocks": list(hit.block_ids),
                              "node": h_of(hit.node)}
            elif kind == "insert":
                al = []
                try:
                    for _ in range(op["nb"]):
                        al.append(cache.alloc_block())
                except oom_error:
                    for b in al:
                        cache._free_block(b)
                    got["alloc"] = al
                    raise
                got["alloc"] = al
                par = op["parent"]
                node = cache.insert(op["tokens"], op["prefix_blocks"] + al,
                                    parent=handles[par] if par else None)
                got["res"] = h_of(node)
            elif kind == "acquire":
                cache.acquire(handles[op["node"]])
            elif kind == "release":
                cache.release(handles[op["node"]])
            elif kind == "evict":
                got["res"] = cache.evict(op["n"])
            elif kind == "ensure_free":
                cache.ensure_free(op["n"])
            elif kind == "alloc":
                got["res"] = cache.alloc_block()
            elif kind == "free":
                cache._free_block(op["bid"])
        except Exception as e:  # noqa: BLE001
            got["error"] = ("OutOfKVCacheError" if isinstance(e, oom_error)
                            else type(e).__name__)
        for key in ("res", "alloc", "error"):
            if op.get(key) != got.get(key):
                bad.append(f"op {i} {kind}: {key} expected {op.get(key)} got {got.get(key)}")
        after = {"free": list(cache._free.keys()), "stats": cache.stats()}
        if after != op["after"]:
            bad.append(f"op {i} {kind}: state expected {op['after']} got {after}")
        if len(bad) > 5:
            break
    if not bad and tree_sig(cache._root) != fixture["final_tree"]:
        bad.append("final tree differs")
    return bad
