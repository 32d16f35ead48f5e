"""NumPy <-> CUDA tensor plumbing for the drop-in API.

The reference passes NumPy arrays (float32, float64, or ml_dtypes.bfloat16
for bf16 pools).  These helpers move them to the device as torch tensors and
bring float32 / bf16 results back as NumPy arrays for NumPy callers.
"""
from __future__ import annotations

import numpy as np
import torch

try:
    import ml_dtypes
    NP_BF16 = np.dtype(ml_dtypes.bfloat16)
except ImportError:  # pragma: no cover - present in this image
    ml_dtypes = None
    NP_BF16 = None


def torch_dtype(dt) -> torch.dtype:
    """Map a NumPy / ml_dtypes / torch / string dtype to a torch dtype."""
    if isinstance(dt, torch.dtype):
        return dt
    if isinstance(dt, str):
        key = dt.lower()
        table = {"float32": torch.float32, "fp32": torch.float32, "f32": torch.float32,
                 "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
                 "float16": torch.float16, "fp16": torch.float16, "f16": torch.float16}
        if key in table:
            return table[key]
    npdt = np.dtype(dt)
    if NP_BF16 is not None and npdt == NP_BF16:
        return torch.bfloat16
    if npdt == np.float32:
        return torch.float32
    if npdt == np.float16:
        return torch.float16
    raise TypeError(f"unsupported KV dtype {dt!r} (float32, bfloat16 or float16)")


def numpy_dtype(dt: torch.dtype):
    if dt == torch.float32:
        return np.dtype(np.float32)
    if dt == torch.float16:
        return np.dtype(np.float16)
    if dt == torch.bfloat16 and NP_BF16 is not None:
        return NP_BF16
    raise TypeError(f"no NumPy dtype for {dt}")


def to_device(x, device: torch.device, *, float_only: bool = True) -> torch.Tensor:
    """Copy a NumPy array / torch tensor to ``device`` as a contiguous tensor.

    float64 is narrowed to float32 (the reference's pools are float32 or
    narrower); ml_dtypes.bfloat16 arrays become torch.bfloat16 bit-for-bit.
    """
    if isinstance(x, torch.Tensor):
        t = x
        if float_only and t.dtype == torch.float64:
            t = t.to(torch.float32)
        return t.to(device, non_blocking=True).contiguous()
    a = np.asarray(x)
    if NP_BF16 is not None and a.dtype == NP_BF16:
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    elif float_only and a.dtype == np.float64:
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    elif float_only and a.dtype.kind in "iub":
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    else:
        t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(device).contiguous()


def upload(a, device: torch.device) -> torch.Tensor:
    """Host metadata (NumPy) -> device without synchronising the stream: the
    array is staged in pinned memory and copied with ``non_blocking`` on the
    current stream (torch keeps the pinned buffer until the copy has run), so
    the host can plan the next step while the device still runs this one."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if torch.device(device).type != "cuda":
        return t
    return t.pin_memory().to(device, non_blocking=True)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    """Device tensor -> NumPy (bf16 as ml_dtypes.bfloat16)."""
    if t.dtype == torch.bfloat16:
        if NP_BF16 is None:
            raise TypeError("ml_dtypes is needed to return bfloat16 NumPy arrays")
        return t.detach().view(torch.int16).cpu().numpy().view(NP_BF16)
    return t.detach().cpu().numpy()
