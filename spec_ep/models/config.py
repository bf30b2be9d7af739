"""Model configurations (Qwen3-MoE family shapes)."""
from __future__ import annotations

from dataclasses import asdict, dataclass


@dataclass
class MoEModelConfig:
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_layers: int = 48
    num_heads: int = 32
    num_kv_heads: int = 4
    head_dim: int = 128
    moe_intermediate_size: int = 768
    num_experts: int = 128
    top_k: int = 8
    norm_topk_prob: bool = True
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02

    def to_dict(self):
        return asdict(self)

    @property
    def qkv_width(self):
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim

    def param_counts(self):
        """(total, expert) parameter counts of the full (unsharded) model."""
        H, I, E = self.hidden_size, self.moe_intermediate_size, self.num_experts
        attn = H * self.qkv_width + self.num_heads * self.head_dim * H + 2 * self.head_dim
        expert = E * 3 * H * I
        per_layer = attn + expert + E * H + 2 * H
        emb = self.vocab_size * H * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * per_layer + emb + H, self.num_layers * expert


PRESETS = {
    # Qwen3-30B-A3B (transformers Qwen3MoeConfig defaults for that checkpoint)
    "qwen3-30b-a3b": MoEModelConfig(),
    # Qwen3-235B-A22B MoE layer shape (hidden 4096, 64 q / 4 kv heads, inter 1536)
    "qwen3-235b-a22b": MoEModelConfig(hidden_size=4096, num_layers=94, num_heads=64, num_kv_heads=4,
                                      moe_intermediate_size=1536),
    # small shapes for tests and smoke runs
    "tiny": MoEModelConfig(vocab_size=4096, hidden_size=512, num_layers=2, num_heads=4, num_kv_heads=2,
                           moe_intermediate_size=256, num_experts=8, top_k=2),
}


def get_config(name: str, **overrides) -> MoEModelConfig:
    cfg = MoEModelConfig(**PRESETS[name].to_dict())
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg
