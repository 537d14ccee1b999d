"""Test infrastructure: the parity oracle (the reference's CPU path, compiled from its sources, and a CPU restatement).
Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg."""
