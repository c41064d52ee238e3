"""CPU oracle of modelcore's KV-cache decode path -- test infrastructure, never product code.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package.
"""
