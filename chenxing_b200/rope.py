"""Rotary position embedding tables and the fused RoPE + KV append.

The reference rotates Q and K in NumPy right before ``write_layer``
(``chenxing/model/transformer.py:84-87`` via ``apply_rope``,
``chenxing/core/tensor.py:129-180``) with cos / sin tables from
``build_rope_cache`` (``tensor.py:80-121``).  ``RopeTables`` builds the same
tables on the host (same float64 arithmetic, cast to fp32) and keeps them in
device memory; ``RadixPagedKVCache.append_rope`` / ``cx_kv_append_rope``
then rotates K while scattering it into the pool, copies V, and rotates Q
into a separate output in the same launch.  Every rotated element is the
fp32 product-sum the reference computes (no fused multiply-add), so fp32
results are bit-identical and bf16 pools hold its round-to-nearest-even.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib

__all__ = ["build_rope_cache", "RopeTables"]


def build_rope_cache(seq_len: int, head_dim: int, base: float = 10000.0, *,
                     scaling_factor: float = 1.0, original_max_pos: int = 4096,
                     beta_fast: float = 32.0, beta_slow: float = 1.0):
    """cos, sin float32 (seq_len, head_dim) — the reference's tables: plain RoPE
    frequencies base^(-2i/d), or with scaling_factor != 1 the YaRN ramp that
    keeps high frequencies and divides low ones by the factor."""
    half = head_dim // 2
    inv_freq = base ** (-np.arange(0, half, dtype=np.float64) * 2.0 / head_dim)
    if scaling_factor != 1.0:
        two_log_base = 2 * np.log(base)
        low = head_dim * np.log(original_max_pos / (beta_fast * 2 * np.pi)) / two_log_base
        high = head_dim * np.log(original_max_pos / (beta_slow * 2 * np.pi)) / two_log_base
        low, high = max(float(np.floor(low)), 0.0), min(float(np.ceil(high)), half - 1.0)
        ramp = np.arange(half, dtype=np.float64) - low
        ramp = np.clip(ramp / max(high - low, 1e-9), 0.0, 1.0)
        inv_freq = inv_freq * (1 - ramp) + (inv_freq / scaling_factor) * ramp
    angles = np.outer(np.arange(seq_len, dtype=np.float64), inv_freq)
    angles = np.concatenate([angles, angles], axis=-1)
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


class RopeTables:
    """Device-resident cos / sin tables of one model's RoPE configuration."""

    def __init__(self, max_positions: int, head_dim: int, base: float = 10000.0, *,
                 scaling_factor: float = 1.0, original_max_pos: int = 4096,
                 beta_fast: float = 32.0, beta_slow: float = 1.0, interleaved: bool = False,
                 device=None, tables=None) -> None:
        self.device = _lib.require_cuda(device)
        if tables is None:
            tables = build_rope_cache(max_positions, head_dim, base,
                                      scaling_factor=scaling_factor,
                                      original_max_pos=original_max_pos,
                                      beta_fast=beta_fast, beta_slow=beta_slow)
        cos, sin = (np.ascontiguousarray(t, dtype=np.float32) for t in tables)
        if cos.shape != sin.shape or cos.ndim != 2 or cos.shape[1] != head_dim:
            raise ValueError("cos / sin tables must both be (positions, head_dim)")
        self.head_dim = int(head_dim)
        self.rows = int(cos.shape[0])
        self.interleaved = bool(interleaved)
        self.cos = torch.from_numpy(cos).to(self.device)
        self.sin = torch.from_numpy(sin).to(self.device)
