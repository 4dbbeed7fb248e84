"""CPU oracle for the CSA / DSV4 decode path — TEST INFRASTRUCTURE, not product.

Numpy restatements of ypd666/CSAHCA's PyTorch reference math
(hybrid_attention/reference.py, hybrid_attention/dsv4_correctness.py), pinned
against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  Only `tests/`, `__graft_entry__.smoke()` and the
CPU-baseline legs of `bench.py` may import this package; the CUDA product path
never calls it and fails loudly when its extension is missing.
"""
