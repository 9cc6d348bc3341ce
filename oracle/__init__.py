"""CPU oracle of the MoE expert-layer forward path (test infrastructure only):
moe_oracle (numpy, the checker) and torch_ref (the reference's torch chain
restated on the CPU, the timed CPU baseline).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs;
never by the product package.
"""
