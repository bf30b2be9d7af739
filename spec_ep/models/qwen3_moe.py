"""Qwen3-MoE-shaped decoder on the sm_100a ops, with expert parallelism.

Per layer:
    h = RMSNorm(x)
    qkv = h @ W_qkv^T                              (one fused projection, tcgen05 GEMM)
    q, k, v = qk_norm_rope(qkv)                    (per-head RMSNorm + RoPE, one kernel)
    x = x + attn(q, k, v) @ W_o^T                  (causal GQA)
    h = RMSNorm(x)
    w, e = router_topk(h @ W_router^T)             (softmax / top-k / renorm kernel)
    x = x + MoE(h; e, w)                           (EP dispatch -> tcgen05 GEMMs -> combine;
                                                    the residual add is folded into the
                                                    source-side reduction)

Expert weights use the transformers layout (``gate_up_proj [E, 2I, H]``,
``down_proj [E, H, I]``) restricted to this rank's local experts; see
``spec_ep.integrations.hf_qwen`` for loading HF checkpoints.

Reference parity: the reference's model path runs HF Qwen3.5-MoE under DeepSpeed AutoEP,
forward only (scripts/ds_moe.py:26-61, :145-174); this module is the trainable
equivalent with the dispatch of src/rbd.py wired into the MoE block.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops.attention import causal_gqa_attention
from ..ops.linear import dense_fwd, linear
from ..ops.loss import lm_head_xent
from ..ops.norm import add_rms_norm, rms_norm, rms_norm_res
from ..ops.rope import qk_norm_rope
from ..ops.router import router_topk
from ..parallel.ep import ExpertParallel, ep_moe
from .config import MoEModelConfig


def _normal(shape, std, device, dtype):
    return torch.empty(shape, device=device, dtype=dtype).normal_(0.0, std)


class Qwen3MoeLayer(nn.Module):
    def __init__(self, cfg: MoEModelConfig, ep: ExpertParallel, device, dtype=torch.bfloat16):
        super().__init__()
        H, D, I = cfg.hidden_size, cfg.head_dim, cfg.moe_intermediate_size
        std = cfg.initializer_range
        self.cfg, self.ep = cfg, ep
        self.input_norm = nn.Parameter(torch.ones(H, device=device, dtype=dtype))
        self.w_qkv = nn.Parameter(_normal((cfg.qkv_width, H), std, device, dtype))
        self.q_norm = nn.Parameter(torch.ones(D, device=device, dtype=dtype))
        self.k_norm = nn.Parameter(torch.ones(D, device=device, dtype=dtype))
        self.w_o = nn.Parameter(_normal((H, cfg.num_heads * D), std, device, dtype))
        self.post_norm = nn.Parameter(torch.ones(H, device=device, dtype=dtype))
        self.w_router = nn.Parameter(_normal((cfg.num_experts, H), std, device, dtype))
        G = ep.G
        self.w_gu = nn.Parameter(_normal((G, 2 * I, H), std, device, dtype))
        self.w_d = nn.Parameter(_normal((G, H, I), std, device, dtype))
        for p in (self.w_gu, self.w_d):
            p._sepx_expert = True
        self.grad_sink = None
        self.router_bias = None  # optional selection bias added to the probabilities
        self.router_logit_bias = None  # optional fp32 [E] bias added to the router logits (skew studies)
        self.routing_callback = None  # receives topk expert ids (routing capture)
        self.spec = None  # SpeculativeExperts (speculative replication, inference only)

    def forward(self, x, pos=None):
        cfg = self.cfg
        spec = self.spec
        x_in = x
        if spec is not None:
            if torch.is_grad_enabled() and self.w_gu.requires_grad:
                raise RuntimeError("speculative expert replication is inference-only: run under torch.no_grad()")
            # predict this layer's experts from the incoming residual stream; the replica
            # fetch runs on a side stream while the attention below executes
            spec.speculate(x, self.post_norm, self.w_router, cfg.top_k, cfg.rms_norm_eps, cfg.norm_topk_prob,
                           self.router_bias, self.router_logit_bias)
        # the residual adds and the gradient sums of the residual stream ride in the norm
        # kernels (rms_norm_res, add_rms_norm)
        h, x = rms_norm_res(x, self.input_norm, cfg.rms_norm_eps)
        qkv = linear(h, self.w_qkv)
        q, k, v = qk_norm_rope(qkv, self.q_norm, self.k_norm, cfg.num_heads, cfg.num_kv_heads, cfg.rms_norm_eps,
                               cfg.rope_theta, pos)
        a = causal_gqa_attention(q, k, v)
        x, h = add_rms_norm(x, linear(a, self.w_o), self.post_norm, cfg.rms_norm_eps)
        logits = linear(h, self.w_router).float()
        if self.router_logit_bias is not None:
            logits = logits + self.router_logit_bias
        topk_w, topk_e = router_topk(logits, cfg.top_k, cfg.norm_topk_prob, self.router_bias)
        if self.routing_callback is not None:
            self.routing_callback(topk_e)
        if spec is not None:
            spec.observe(x_in, topk_e)
            return ep_moe(h, topk_e, topk_w, spec.w_gu, spec.w_d, self.ep, None, residual=x, route=spec.tables())
        return ep_moe(h, topk_e, topk_w, self.w_gu, self.w_d, self.ep, self.grad_sink, residual=x)


class Qwen3MoeForCausalLM(nn.Module):
    """Decoder-only MoE LM; ``forward(input_ids, labels)`` returns the mean CE loss."""

    def __init__(self, cfg: MoEModelConfig, ep: ExpertParallel, device=None, dtype=torch.bfloat16):
        super().__init__()
        device = device or ep.device
        self.cfg, self.ep = cfg, ep
        self.embed = nn.Parameter(_normal((cfg.vocab_size, cfg.hidden_size), cfg.initializer_range, device, dtype))
        self.layers = nn.ModuleList([Qwen3MoeLayer(cfg, ep, device, dtype) for _ in range(cfg.num_layers)])
        self.final_norm = nn.Parameter(torch.ones(cfg.hidden_size, device=device, dtype=dtype))
        if cfg.tie_word_embeddings:
            self.lm_head = self.embed
        else:
            self.lm_head = nn.Parameter(_normal((cfg.vocab_size, cfg.hidden_size), cfg.initializer_range, device,
                                                dtype))

    def expert_parameters(self):
        return [p for p in self.parameters() if getattr(p, "_sepx_expert", False)]

    def dense_parameters(self):
        return [p for p in self.parameters() if not getattr(p, "_sepx_expert", False)]

    def set_grad_sink(self, sink):
        for layer in self.layers:
            layer.grad_sink = sink

    def hidden_states(self, input_ids, pos=None):
        x = F.embedding(input_ids.view(-1), self.embed)
        for layer in self.layers:
            x = layer(x, pos)
        return rms_norm(x, self.final_norm, self.cfg.rms_norm_eps)

    def forward(self, input_ids, labels=None, num_valid=None, pos=None):
        h = self.hidden_states(input_ids, pos)
        if labels is None:
            return dense_fwd(h, self.lm_head)
        return lm_head_xent(h, self.lm_head, labels.view(-1), num_valid)
