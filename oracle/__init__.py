"""CPU oracle of the MoE expert-layer forward path (test infrastructure only).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs;
never by the product package.
"""
