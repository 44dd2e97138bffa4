"""TEST INFRASTRUCTURE ONLY -- the CPU checker for the K1 kernels.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import
this package.  The product path (kernel_opt) never does.
"""
