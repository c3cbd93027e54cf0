"""ORACLE -- test infrastructure, not product code.

CPU restatements of the reference's algorithms for the N:M sparse GEMV
decode path, used only as the checker by tests/, by
__graft_entry__.smoke() and by bench.py's cpu_baseline / reference arm.
The product package (spmv_decode_b200) never imports this package.
Pinned against the golden fixtures in tests/golden/, which were produced by
the reference's own code (tests/golden/make_golden.py).
"""
