"""CPU oracle for the RQF scan family — test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this package, and only as the checker (or the timed CPU baseline),
never as the product path.  See oracle/rqf_oracle.c for the restated
reference algorithms and oracle/selective.py for the selective scan.
"""
