"""CPU oracle for the paged-attention path — test infrastructure only.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
the checker or the timed CPU baseline; never by the product path.
"""
