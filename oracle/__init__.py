"""CPU oracle for the Chenxing KV-cache hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in plain NumPy, the reference algorithms that the CUDA
path in ``chenxing_b200`` replaces:

* ``oracle.attention``  — blocked online-softmax attention, the naive
  full-softmax kernel, GQA head expansion and causal / sliding-window masks
  (reference ``chenxing/core/attention.py`` and ``chenxing/core/tensor.py``).
* ``oracle.radix_kv``   — the physical block pool (FIFO free list, per-token
  ``write_layer`` scatter, ``read_layer`` gather) and the logical radix prefix
  tree (reference ``chenxing/engine/radix_kv.py``).
* ``oracle.paged``      — the per-sequence decode / verify path exactly as the
  reference model drives it (write -> read -> attention), plus the block-table
  growth and speculative-rollback metadata rules of the reference engine.

Pinning: every function here is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``), see
``tests/test_oracle_golden.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package, and only as the checker / the timed CPU
baseline.  The product path (``chenxing_b200``) never imports it and has no
CPU fallback.
"""
