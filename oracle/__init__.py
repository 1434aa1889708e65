"""Parity oracles for the dense matmul path (test infrastructure only).

Nothing in the product (cmp_ext_b200/, cmpext3.py) imports this package; only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
"""
