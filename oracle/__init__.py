"""CPU oracle for manifesto's dtype/convert + fused-elementwise hot path.

TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this package, and only as the checker or the
timed CPU baseline; the product package (manifesto_b200) never does.
"""
