"""TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's GEMM oracle.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
import this package, and only as the checker or the timed CPU baseline -- never as the
product path.  The product path is libtempo_sm100.so and fails loudly without it.
"""
