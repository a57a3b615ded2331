"""CPU oracle for the GEMM hot path — test infrastructure only.

Imported only by tests/, __graft_entry__.smoke() and bench.py (CPU baseline and the
reference arm). The product package never imports it.
"""
