"""CPU oracle of the MoE MLP hot path -- test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this package, and only as the checker / reported CPU baseline.  The
product (triton-variable-moe_b200/) never imports it.
"""
