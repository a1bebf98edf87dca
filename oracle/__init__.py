"""CPU oracle for the paged-attention hot path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs;
never by the product package (gb10-attn_b200/pa_b200), which has no CPU path.
"""
