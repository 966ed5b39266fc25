"""Test infrastructure: CPU restatement of the reference blend prefill (the checker).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.
"""
