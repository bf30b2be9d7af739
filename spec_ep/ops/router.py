"""Router: softmax over experts, top-k, optional renormalisation (sm_100a kernel).

Matches transformers' Qwen3-MoE router (softmax in fp32, ``norm_topk_prob``). The
optional ``bias`` shifts only the *selection* scores (not the returned weights); the
synthetic-skew benchmarks use it to make expert popularity follow a Zipf law.
"""
from __future__ import annotations

import torch

from ._ext import load


class _RouterTopK(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, k, renorm, bias):
        C = load()
        T, E = logits.shape
        topk_e = torch.empty(T, k, device=logits.device, dtype=torch.int32)
        topk_w = torch.empty(T, k, device=logits.device, dtype=torch.float32)
        probs = torch.empty(T, E, device=logits.device, dtype=torch.float32)
        C.router_topk(logits.contiguous(), bias, k, renorm, topk_e, topk_w, probs)
        ctx.save_for_backward(probs, topk_e)
        ctx.renorm = renorm
        ctx.mark_non_differentiable(topk_e)
        return topk_w, topk_e

    @staticmethod
    def backward(ctx, dw, _de):
        probs, topk_e = ctx.saved_tensors
        dlogits = torch.empty_like(probs)
        load().router_bwd(probs, topk_e, dw.contiguous().float(), ctx.renorm, dlogits)
        return dlogits, None, None, None


def router_topk(logits: torch.Tensor, k: int, renorm: bool = True, bias: torch.Tensor | None = None):
    """Returns (topk_w [T, k] fp32, topk_e [T, k] int32) from fp32 router logits."""
    return _RouterTopK.apply(logits.float(), k, renorm, bias)


def router_topk_reference(logits, k, renorm=True, bias=None):
    p = torch.softmax(logits.float(), -1)
    score = p if bias is None else p + bias
    idx = score.topk(k, -1).indices
    w = p.gather(-1, idx)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w, idx.int()
