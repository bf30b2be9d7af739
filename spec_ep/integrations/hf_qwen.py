"""transformers Qwen3-MoE integration.

* ``SepxQwen3MoeBlock`` is a drop-in replacement for transformers'
  ``Qwen3MoeSparseMoeBlock`` (``mlp`` of every decoder layer): the router runs on the
  sm_100a top-k kernel and the experts on the fused expert-parallel layer, holding only
  this rank's experts (``gate_up_proj [E, 2I, H]`` / ``down_proj [E, H, I]`` slices).
* ``swap_moe_blocks(hf_model, ep)`` replaces every such block in place.
* ``from_hf`` / ``to_hf_state_dict`` convert weights between a transformers
  ``Qwen3MoeForCausalLM`` and ``spec_ep.models.qwen3_moe.Qwen3MoeForCausalLM`` (HF
  safetensors stays the checkpoint format).

Reference parity: the reference swaps HF MoE blocks for DeepSpeed's AutoEP layer
(scripts/ds_moe.py:50-61) and runs HF generate in scripts/hf_qwen.py:44-78.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..models.config import MoEModelConfig
from ..ops.router import router_topk
from ..parallel.ep import ExpertParallel, ep_moe


def config_from_hf(hf_cfg) -> MoEModelConfig:
    """MoEModelConfig from a transformers Qwen3MoeConfig (text config)."""
    c = getattr(hf_cfg, "text_config", hf_cfg)
    return MoEModelConfig(
        vocab_size=c.vocab_size, hidden_size=c.hidden_size, num_layers=c.num_hidden_layers,
        num_heads=c.num_attention_heads, num_kv_heads=c.num_key_value_heads,
        head_dim=getattr(c, "head_dim", c.hidden_size // c.num_attention_heads),
        moe_intermediate_size=c.moe_intermediate_size, num_experts=c.num_experts, top_k=c.num_experts_per_tok,
        norm_topk_prob=c.norm_topk_prob, rope_theta=getattr(c, "rope_theta", None) or c.rope_parameters["rope_theta"],
        rms_norm_eps=c.rms_norm_eps, tie_word_embeddings=getattr(c, "tie_word_embeddings", False),
        initializer_range=getattr(c, "initializer_range", 0.02))


def _local_ids(ep: ExpertParallel):
    if ep.placement is not None:
        return ep.placement.local_experts[ep.rank]
    return list(range(ep.rank * ep.G, (ep.rank + 1) * ep.G))


class SepxQwen3MoeBlock(nn.Module):
    """Qwen3-MoE sparse block on the fused B200 expert-parallel layer."""

    def __init__(self, gate_weight: torch.Tensor, gate_up_proj: torch.Tensor, down_proj: torch.Tensor,
                 top_k: int, norm_topk_prob: bool, ep: ExpertParallel):
        super().__init__()
        self.ep, self.top_k, self.norm_topk_prob = ep, top_k, norm_topk_prob
        local = _local_ids(ep)
        dev, dt = ep.device, torch.bfloat16
        self.gate_weight = nn.Parameter(gate_weight.detach().to(dev, dt).contiguous())
        self.gate_up_proj = nn.Parameter(gate_up_proj.detach()[local].to(dev, dt).contiguous())
        self.down_proj = nn.Parameter(down_proj.detach()[local].to(dev, dt).contiguous())
        for p in (self.gate_up_proj, self.down_proj):
            p._sepx_expert = True
        self.grad_sink = None

    @classmethod
    def from_hf_block(cls, block, ep: ExpertParallel):
        return cls(block.gate.weight, block.experts.gate_up_proj, block.experts.down_proj, block.gate.top_k,
                   block.gate.norm_topk_prob, ep)

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        logits = torch.nn.functional.linear(x, self.gate_weight).float()
        w, e = router_topk(logits, self.top_k, self.norm_topk_prob)
        out = ep_moe(x, e, w, self.gate_up_proj, self.down_proj, self.ep, self.grad_sink)
        return out.view(shape).to(hidden_states.dtype)


class SepxQwen3_5MoeBlock(SepxQwen3MoeBlock):
    """Qwen3.5-MoE block (the reference's model family, scripts/ds_moe.py:15,28): routed
    experts on the fused EP layer plus the sigmoid-gated shared expert, which stays a
    dense, replicated transformers module."""

    def __init__(self, block, ep: ExpertParallel):
        super().__init__(block.gate.weight, block.experts.gate_up_proj, block.experts.down_proj, block.gate.top_k,
                         block.gate.norm_topk_prob, ep)
        self.shared_expert = block.shared_expert
        self.shared_expert_gate = block.shared_expert_gate

    def forward(self, hidden_states):
        shape = hidden_states.shape
        flat = hidden_states.reshape(-1, shape[-1])
        shared = torch.sigmoid(self.shared_expert_gate(flat)) * self.shared_expert(flat)
        return super().forward(hidden_states) + shared.view(shape).to(hidden_states.dtype)


def swap_moe_blocks(hf_model: nn.Module, ep: ExpertParallel) -> int:
    """Replace every Qwen3-MoE / Qwen3.5-MoE sparse block of ``hf_model`` in place.

    Returns the number of blocks replaced.
    """
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    try:
        from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock
    except ImportError:  # older transformers
        Qwen3_5MoeSparseMoeBlock = ()
    n = 0
    for module in list(hf_model.modules()):
        for name, child in list(module.named_children()):
            if Qwen3_5MoeSparseMoeBlock and isinstance(child, Qwen3_5MoeSparseMoeBlock):
                setattr(module, name, SepxQwen3_5MoeBlock(child, ep))
                n += 1
            elif isinstance(child, Qwen3MoeSparseMoeBlock):
                setattr(module, name, SepxQwen3MoeBlock.from_hf_block(child, ep))
                n += 1
    return n


@torch.no_grad()
def from_hf(hf_model, model) -> None:
    """Copy weights of a transformers Qwen3MoeForCausalLM into a spec_ep model
    (this rank's experts only)."""
    hf = hf_model.model if hasattr(hf_model, "model") else hf_model
    local = _local_ids(model.ep)
    model.embed.copy_(hf.embed_tokens.weight)
    model.final_norm.copy_(hf.norm.weight)
    if not model.cfg.tie_word_embeddings:
        model.lm_head.copy_(hf_model.lm_head.weight)
    for layer, hl in zip(model.layers, hf.layers):
        a = hl.self_attn
        layer.w_qkv.copy_(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0))
        layer.w_o.copy_(a.o_proj.weight)
        layer.q_norm.copy_(a.q_norm.weight)
        layer.k_norm.copy_(a.k_norm.weight)
        layer.input_norm.copy_(hl.input_layernorm.weight)
        layer.post_norm.copy_(hl.post_attention_layernorm.weight)
        layer.w_router.copy_(hl.mlp.gate.weight)
        layer.w_gu.copy_(hl.mlp.experts.gate_up_proj[local])
        layer.w_d.copy_(hl.mlp.experts.down_proj[local])


@torch.no_grad()
def to_hf_state_dict(model, gather_experts=None) -> dict:
    """transformers-named state dict of a spec_ep model. ``gather_experts(t)`` must return the
    full ``[E, ...]`` expert tensor from this rank's shard (identity on one GPU)."""
    cfg = model.cfg
    q = cfg.num_heads * cfg.head_dim
    kv = cfg.num_kv_heads * cfg.head_dim
    g = gather_experts or (lambda t: t)
    sd = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.final_norm}
    if not cfg.tie_word_embeddings:
        sd["lm_head.weight"] = model.lm_head
    for i, l in enumerate(model.layers):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = l.w_qkv[:q]
        sd[p + "self_attn.k_proj.weight"] = l.w_qkv[q:q + kv]
        sd[p + "self_attn.v_proj.weight"] = l.w_qkv[q + kv:]
        sd[p + "self_attn.o_proj.weight"] = l.w_o
        sd[p + "self_attn.q_norm.weight"] = l.q_norm
        sd[p + "self_attn.k_norm.weight"] = l.k_norm
        sd[p + "input_layernorm.weight"] = l.input_norm
        sd[p + "post_attention_layernorm.weight"] = l.post_norm
        sd[p + "mlp.gate.weight"] = l.w_router
        sd[p + "mlp.experts.gate_up_proj"] = g(l.w_gu)
        sd[p + "mlp.experts.down_proj"] = g(l.w_d)
    return {k: v.detach() for k, v in sd.items()}


def random_hf_model(num_layers=2, hidden=512, experts=8, top_k=2, inter=256, vocab=4096, heads=4, kv_heads=2,
                    seed=0, dtype=torch.bfloat16):
    """A small random-init transformers Qwen3MoeForCausalLM (no download)."""
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen3MoeConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=4 * hidden,
                         moe_intermediate_size=inter, num_hidden_layers=num_layers, num_attention_heads=heads,
                         num_key_value_heads=kv_heads, head_dim=128, num_experts=experts, num_experts_per_tok=top_k,
                         norm_topk_prob=True, decoder_sparse_step=1, mlp_only_layers=[], rope_theta=1e6,
                         max_position_embeddings=8192, tie_word_embeddings=False)
    m = Qwen3MoeForCausalLM(cfg).to(dtype)
    with torch.no_grad():  # HF leaves the router at zeros; give it some signal
        for layer in m.model.layers:
            layer.mlp.gate.weight.normal_(0, 0.02)
            layer.mlp.experts.gate_up_proj.normal_(0, 0.02)
            layer.mlp.experts.down_proj.normal_(0, 0.02)
    return m
