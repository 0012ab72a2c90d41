"""The NumPy oracle of the Kernel IR semantics.

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this package, as the checker of the CUDA path; the product (ptxgen) never does.
"""
