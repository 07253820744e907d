"""f64 CPU oracle for the GDR path -- test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker or the timed CPU reference; the CUDA
library never routes through it.
"""
