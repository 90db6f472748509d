"""B200-native MoE MLP hot path (drop-in for triton_moe)."""
