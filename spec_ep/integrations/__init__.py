"""Integrations: transformers Qwen3-MoE / Qwen3.5-MoE blocks, DeepSpeed-style configs."""
