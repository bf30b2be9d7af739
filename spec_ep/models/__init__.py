"""Model definitions (Qwen3-MoE family) on the sm_100a ops."""
