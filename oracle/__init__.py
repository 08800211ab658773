"""CPU checkers for the coat_b200 kernels.

TEST INFRASTRUCTURE ONLY.  Nothing in the `coat_b200` package imports this
package; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference legs do, and only as the checker or the timed CPU baseline.
"""
