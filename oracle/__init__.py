"""Test infrastructure only: the CPU oracle for the int4 weight-only matmul path (see oracle.py)."""
