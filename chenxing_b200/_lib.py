"""ctypes binding of libcxkv.so (the C ABI declared in include/cxkv.h).

The shared library is built in-tree by ``chenxing_b200.build`` and loaded
lazily on first use.  There is no CPU fallback: if the library or a CUDA
device is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcxkv.so")

# status codes (cxkv.h)
CX_OK, CX_ERR_RANGE, CX_ERR_SHAPE, CX_ERR_CUDA, CX_ERR_DTYPE, CX_ERR_UNSUPPORTED, \
    CX_ERR_WORKSPACE = range(7)
# element types
CX_F32, CX_BF16, CX_F16 = 0, 1, 2
# device flag bits
DEV_FLAG_NAMES = {1: "bad slot", 2: "bad block id", 4: "context longer than its block table",
                  8: "pipeline wait timeout", 16: "bad query length",
                  32: "RoPE position outside the table"}

EXPORTS = ("cx_version", "cx_last_error", "cx_device_error", "cx_kv_append", "cx_kv_gather",
           "cx_block_copy", "cx_paged_workspace_bytes", "cx_paged_decode", "cx_paged_verify",
           "cx_attention_dense", "cx_paged_decode_static", "cx_paged_kernel_kind",
           "cx_kv_append_rope", "cx_set_wait_limit_ns")
KERNEL_KINDS = {0: "generic", 1: "mma", 2: "tcgen05", 3: "fma"}


class CxPool(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("n_layers", ctypes.c_int64), ("n_blocks", ctypes.c_int64),
                ("block_size", ctypes.c_int64), ("n_kv_heads", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("dtype", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class CxAttnBatch(ctypes.Structure):
    _fields_ = [("block_tables", ctypes.c_void_p), ("table_stride", ctypes.c_int64),
                ("ctx_lens", ctypes.c_void_p), ("q_start", ctypes.c_void_p),
                ("batch", ctypes.c_int64), ("max_q_len", ctypes.c_int64),
                ("n_q_heads", ctypes.c_int64), ("scale", ctypes.c_float),
                ("reserved", ctypes.c_int32), ("window", ctypes.c_int64)]


class CxError(RuntimeError):
    """A libcxkv call returned a non-OK status."""


_lib = None
_lock = threading.Lock()

_VP, _I64, _I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
_SIGS = {
    "cx_version": ([], ctypes.c_char_p),
    "cx_last_error": ([], ctypes.c_char_p),
    "cx_device_error": ([_VP, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "cx_kv_append": ([ctypes.POINTER(CxPool), _I64, _VP, _VP, _I32, _VP, _I64, _VP, _VP, _VP,
                      _I64, _VP], ctypes.c_int),
    "cx_kv_gather": ([ctypes.POINTER(CxPool), _I64, _VP, _I64, _VP, _VP, _VP], ctypes.c_int),
    "cx_block_copy": ([ctypes.POINTER(CxPool), _VP, _VP, _I64, _I64, _VP], ctypes.c_int),
    "cx_paged_workspace_bytes": ([ctypes.POINTER(CxPool), ctypes.POINTER(CxAttnBatch)],
                                 ctypes.c_size_t),
    "cx_paged_decode": ([ctypes.POINTER(CxPool), _I64, ctypes.POINTER(CxAttnBatch), _VP, _I32,
                         _VP, _VP, ctypes.c_size_t, _I32, _VP], ctypes.c_int),
    "cx_paged_verify": ([ctypes.POINTER(CxPool), _I64, ctypes.POINTER(CxAttnBatch), _VP, _I32,
                         _VP, _VP, ctypes.c_size_t, _I32, _VP], ctypes.c_int),
    "cx_attention_dense": ([_VP, _I32, _VP, _VP, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                            _I32, _I64, _VP, ctypes.c_float, _VP, _VP], ctypes.c_int),
    "cx_paged_decode_static": ([ctypes.POINTER(CxPool), _I64, ctypes.POINTER(CxAttnBatch), _VP,
                                _I32, _VP, _VP], ctypes.c_int),
    "cx_paged_kernel_kind": ([ctypes.POINTER(CxPool), ctypes.POINTER(CxAttnBatch), _I32, _I32],
                             ctypes.c_int),
    "cx_set_wait_limit_ns": ([ctypes.c_uint64], None),
    "cx_kv_append_rope": ([ctypes.POINTER(CxPool), _I64, _VP, _VP, _I32, _VP, _VP, _I64, _VP, _VP,
                           _I64, _I32, _VP, _I64, _VP, _I32, _VP], ctypes.c_int),
}


def load_library(path: str = LIB_PATH):
    """Load libcxkv.so (no GPU needed) and declare every exported signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise CxError(f"{path} is not built; run chenxing_b200.build.build()")
        lib = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def lib():
    return _lib if _lib is not None else load_library()


def check(rc: int, what: str) -> None:
    if rc == CX_OK:
        return
    msg = (lib().cx_last_error() or b"").decode(errors="replace")
    if rc == CX_ERR_RANGE:
        raise IndexError(f"{what}: {msg}")
    if rc in (CX_ERR_SHAPE, CX_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    if rc == CX_ERR_DTYPE:
        raise TypeError(f"{what}: {msg}")
    raise CxError(f"{what} failed with status {rc}: {msg}")


def require_cuda(device=None) -> torch.device:
    if not torch.cuda.is_available():
        raise CxError("chenxing_b200 needs a CUDA device (B200, sm_100a); none is visible")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    if dev.type != "cuda":
        raise CxError(f"chenxing_b200 runs on CUDA devices only, got {dev}")
    return dev


def cx_dtype(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return CX_F32
    if dt == torch.bfloat16:
        return CX_BF16
    if dt == torch.float16:
        return CX_F16
    raise TypeError(f"unsupported element type {dt}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_flags(clear: bool = True, device=None) -> int:
    """Read (and clear) the library's device-side error flag word."""
    out = ctypes.c_uint32(0)
    check(lib().cx_device_error(stream_ptr(device), int(clear), ctypes.byref(out)),
          "cx_device_error")
    return int(out.value)


def describe_flags(flags: int) -> str:
    return ", ".join(n for bit, n in DEV_FLAG_NAMES.items() if flags & bit) or "none"
