"""Mask marker shared with the reference (chenxing/core/tensor.py:183-186)."""
from __future__ import annotations

from dataclasses import dataclass

__all__ = ["CausalMask", "AttentionMask"]


@dataclass(frozen=True)
class CausalMask:
    """Causal (lower-triangular) attention with optional sliding window.

    Query row ``i`` of ``sq`` rows over ``sk`` keys sits at position
    ``i + sk - sq`` and attends key ``j`` iff ``j <= pos`` and, with a window
    ``w``, ``j + w > pos`` (chenxing/core/attention.py:75-80).
    """
    sliding_window: int | None = None


AttentionMask = object
