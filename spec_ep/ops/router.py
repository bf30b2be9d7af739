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


class _RouterFront(torch.autograd.Function):
    """Router projection + softmax / top-k (+ routing tables) in one tcgen05 GEMM launch."""

    @staticmethod
    def forward(ctx, h, w, k, renorm, sel_bias, logit_bias, e2r, e2l):
        from .linear import _rows_offsets

        C = load()
        T = h.shape[0]
        dev = h.device
        hc = h.contiguous()
        probs = torch.empty(T, 128, device=dev, dtype=torch.float32)
        topk_e = torch.empty(T, k, device=dev, dtype=torch.int32)
        topk_w = torch.empty(T, k, device=dev, dtype=torch.float32)
        dst = meta = None
        if e2r is not None:
            dst = torch.empty(T, k, device=dev, dtype=torch.int32)
            meta = torch.empty(T, k, device=dev, dtype=torch.int32)
        C.gemm_router(hc, w.contiguous(), _rows_offsets(T, dev), logit_bias, sel_bias, k, renorm, e2r, e2l, probs,
                      topk_e, topk_w, dst, meta, None)
        ctx.save_for_backward(hc, w, probs, topk_e)
        ctx.renorm = renorm
        ctx.mark_non_differentiable(topk_e)
        if dst is None:
            return topk_w, topk_e
        ctx.mark_non_differentiable(dst, meta)
        return topk_w, topk_e, dst, meta

    @staticmethod
    def backward(ctx, dw, *_):
        from .linear import dense_dgrad, dense_wgrad

        h, w, probs, topk_e = ctx.saved_tensors
        dlogits = torch.empty_like(probs)
        load().router_bwd(probs, topk_e, dw.contiguous().float(), ctx.renorm, dlogits)
        g = dlogits.to(torch.bfloat16)  # the gradient of the bf16 logits
        dh = dense_dgrad(g, w) if ctx.needs_input_grad[0] else None
        dwr = dense_wgrad(g, h) if ctx.needs_input_grad[1] else None
        return dh, dwr, None, None, None, None, None, None


def router_front(h: torch.Tensor, w: torch.Tensor, k: int, renorm: bool = True, sel_bias=None, logit_bias=None,
                 tables=None):
    """The MoE router from the hidden states in one launch: ``h [T, H] @ w [128, H].T``
    rounded to bf16 (plus ``logit_bias``), softmax, top-k (selection on the probabilities
    plus ``sel_bias``), renormalisation. Returns ``(topk_w, topk_e)`` or, with
    ``tables = (e2r, e2l)`` (expert -> rank, local slot), ``(topk_w, topk_e, dst, meta)``
    for the expert-parallel dispatch. 128 experts, hidden a multiple of 64."""
    e2r, e2l = tables if tables is not None else (None, None)
    f32 = lambda b: None if b is None else b.detach().float().contiguous()  # noqa: E731
    return _RouterFront.apply(h, w, k, renorm, f32(sel_bias), f32(logit_bias), e2r, e2l)


def router_front_supported(w: torch.Tensor, h: torch.Tensor) -> bool:
    """Shapes the fused router front takes (otherwise: projection, then router_topk)."""
    return w.dim() == 2 and w.shape[0] == 128 and h.shape[-1] % 64 == 0 and h.dtype == torch.bfloat16


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
