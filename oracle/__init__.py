"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the W4A8 hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this package.  It restates the reference's algorithm on the CPU (numpy, torch CPU
and the C library built from w4a8_oracle.c) to check the CUDA library and to time
the reference's own CPU path; the product never calls it.
"""
