"""chenxing_b200 — B200-native (sm_100a) KV-cache hot path for Chenxing.

Drop-in replacements for the reference's ``chenxing.engine.radix_kv`` and
``chenxing.core.attention`` interfaces, with the block pool in HBM and every
data-path operation a hand-written CUDA kernel behind the C ABI of
``libcxkv.so`` (``include/cxkv.h``).  Importing the package needs no GPU; the
library is loaded on first use and there is no CPU fallback.
"""
from .attention import flash_attention, gqa_expand, naive_attention
from .batch import PagedBatch, decode_batch, slot_mapping, verify_batch
from .engine import BatchedKVEngine
from .radix_kv import OutOfKVCacheError, PrefixHit, RadixIndex, RadixPagedKVCache
from .rope import RopeTables, build_rope_cache
from .tensor import CausalMask

__all__ = ["RadixPagedKVCache", "RadixIndex", "PrefixHit", "OutOfKVCacheError",
           "flash_attention", "naive_attention", "gqa_expand", "CausalMask",
           "PagedBatch", "decode_batch", "verify_batch", "slot_mapping", "BatchedKVEngine",
           "RopeTables", "build_rope_cache"]
