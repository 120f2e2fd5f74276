"""CPU oracle (test infrastructure only): restatement of the reference's algorithms.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package.
"""
