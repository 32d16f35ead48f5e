"""Rotary position embedding oracle (NumPy) — TEST INFRASTRUCTURE ONLY.

Restates ``chenxing/core/tensor.py``:

* ``rope_tables``  — ``build_rope_cache`` (``tensor.py:80-121``): inverse
  frequencies base^(-2i/d) in float64, optional YaRN ramp between the
  extrapolated and the 1/scale-interpolated frequencies, angles t * f for
  every position, duplicated across the two halves, cos / sin cast to fp32.
* ``rotate``       — ``apply_rope`` (``tensor.py:129-180``) for (T, H, D) rows
  at explicit positions: half-split pairs (j, j + D/2) or interleaved pairs
  (2j, 2j + 1), each output one fp32 product-sum as NumPy evaluates it.
"""
from __future__ import annotations

import numpy as np

__all__ = ["rope_tables", "rotate"]


def rope_tables(n_pos, d, base=10000.0, scaling_factor=1.0, original_max_pos=4096,
                beta_fast=32.0, beta_slow=1.0):
    h = d // 2
    idx = np.arange(0, h, dtype=np.float64)
    inv = base ** (-idx * 2.0 / d)
    if scaling_factor != 1.0:
        lo = d * np.log(original_max_pos / (beta_fast * 2 * np.pi)) / (2 * np.log(base))
        hi = d * np.log(original_max_pos / (beta_slow * 2 * np.pi)) / (2 * np.log(base))
        lo = max(float(np.floor(lo)), 0.0)
        hi = min(float(np.ceil(hi)), h - 1.0)
        w = np.clip((np.arange(h, dtype=np.float64) - lo) / max(hi - lo, 1e-9), 0.0, 1.0)
        inv = inv * (1 - w) + (inv / scaling_factor) * w
    ang = np.outer(np.arange(n_pos, dtype=np.float64), inv)
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rotate(x, cos, sin, positions, interleaved=False):
    """x (T, H, D) float32 -> rotated float32, rows of the tables at positions."""
    x = np.asarray(x, dtype=np.float32)
    c = cos[positions][:, None, :]
    s = sin[positions][:, None, :]
    h = x.shape[-1] // 2
    out = np.empty_like(x)
    if interleaved:
        a, b = x[..., 0::2], x[..., 1::2]
        out[..., 0::2] = a * c[..., :h] - b * s[..., :h]
        out[..., 1::2] = a * s[..., :h] + b * c[..., :h]
        return out
    a, b = x[..., :h], x[..., h:]
    out[..., :h] = a * c[..., :h] + (-b) * s[..., :h]
    out[..., h:] = b * c[..., h:] + a * s[..., h:]
    return out
