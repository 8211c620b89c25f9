"""TEST INFRASTRUCTURE — CPU oracle for specgrove_b200.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package.  It is the checker, never the measured or shipped path.
"""
