"""cx_paged_decode_static: the paged decode entry point that allocates nothing.

It exists for callers that cannot allocate device memory — a serving process
whose HBM is already fully reserved by the block pool and its own allocator,
or a host runtime behind a plain C FFI with no device allocator — and keeps
its scratch in a fixed 8 MiB array inside the library.  These tests call it
through the C ABI and compare it with cx_paged_decode (caller workspace) on
two calls in a row, so the second call runs on scratch left by the first.
Both calls run the same kernel with the same plan and a fixed merge order, so
their outputs must be bit-identical; both are also checked against the CPU
oracle (bf16 pools: max |out - ref| <= 2e-2 * max |ref| per sequence).
Named test_zz_* so pytest collects it last.
"""
import numpy as np
import pytest
import torch

from gpu_cases import BF16_RTOL, PagedCase

pytestmark = pytest.mark.gpu


def _static_decode(case, batch, layer=0):
    from chenxing_b200 import _lib
    out = torch.full((batch.total_q, case.hq, case.d), float("nan"), device="cuda")
    _lib.check(_lib.lib().cx_paged_decode_static(
        case.cache.cx_pool(), layer, batch.c_struct(), case.q_dev.data_ptr(),
        _lib.cx_dtype(case.q_dev.dtype), out.data_ptr(), _lib.stream_ptr()),
        "cx_paged_decode_static")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _same(got, ref, case):
    """Bit-identical to the workspace call, and within tolerance of the oracle."""
    assert np.isfinite(got).all()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), \
        f"static and workspace decode differ (max {float(np.abs(got - ref).max())})"
    case.check(got, rtol=BF16_RTOL)


def test_static_decode_matches_workspace_decode_twice():
    from chenxing_b200 import _lib
    _lib.device_flags(clear=True)
    # call 1: long contexts split across CTAs (exercises the merge tickets)
    a = PagedCase(hq=32, hk=8, d=128, ctx=[9000, 5, 3000, 777], seed=21)
    ref_a = a.run()
    _same(_static_decode(a, a.batch()), ref_a, a)
    # call 2, straight after: another batch shape on the same scratch
    b = PagedCase(hq=16, hk=4, d=64, ctx=[1, 64, 2500, 17, 400, 4097], seed=22,
                  q_dtype=torch.bfloat16)
    ref_b = b.run()
    _same(_static_decode(b, b.batch()), ref_b, b)
    # and the first batch again: nothing stale from call 2 leaks in
    _same(_static_decode(a, a.batch()), ref_a, a)
    assert _lib.device_flags(clear=True) == 0


def test_static_decode_rejects_batches_beyond_its_scratch():
    from chenxing_b200 import PagedBatch, RadixPagedKVCache, _lib
    n = 3000
    cache = RadixPagedKVCache(n, 16, 1, 8, 128, dtype="bfloat16", host_io=False)
    batch = PagedBatch(cache, [[i] for i in range(n)], [1] * n, n_q_heads=32)
    assert int(_lib.lib().cx_paged_workspace_bytes(cache.cx_pool(), batch.c_struct())) > 8 << 20
    q = torch.zeros((n, 32, 128), device="cuda")
    out = torch.zeros((n, 32, 128), device="cuda")
    rc = _lib.lib().cx_paged_decode_static(cache.cx_pool(), 0, batch.c_struct(), q.data_ptr(),
                                           _lib.CX_F32, out.data_ptr(), _lib.stream_ptr())
    assert rc == _lib.CX_ERR_WORKSPACE
    assert b"static area holds" in _lib.lib().cx_last_error()
