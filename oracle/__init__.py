"""CPU oracle for the GDN decode / prefill paths (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package.  It is the checker, never the product path.
"""
