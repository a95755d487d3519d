"""TEST INFRASTRUCTURE ONLY: CPU oracle of the reference's quantised MoE block.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs as the
checker / timed CPU baseline; never by the product package titan_b200.
"""
