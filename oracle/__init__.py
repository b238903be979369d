"""CPU oracle for the MoDA forward: test infrastructure, not part of the library.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
"""
