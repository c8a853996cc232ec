"""Test infrastructure: the CPU oracle (numpy restatements of the reference's
math and a StableHLO interpreter).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg use it; the plugin never does."""
