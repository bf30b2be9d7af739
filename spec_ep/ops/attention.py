"""Causal grouped-query attention (head_dim 128).

q [T, Hq, 128], k/v [T, Hkv, 128] (token-major, as written by the fused q/k-norm+RoPE
kernel) -> out [T, Hq * 128].

``attention_fwd`` / ``attention_bwd`` are the hand-written tcgen05 kernels
(csrc/attention.cu); the forward also returns the per-row log-sum-exp that the backward
uses to recompute the probabilities. ``flash_attention`` wraps both in an autograd
function. The reference runs this op through FlashAttention / SDPA
(benchmark/compute.py:71-96).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ._ext import load


def attention_fwd(q, k, v, scale=None, status=None, two_tile=False, trace=None):
    """tcgen05 forward: returns (o [T, Hq*128] bf16, lse [Hq, T] fp32, natural log).

    ``two_tile`` selects the kernel that runs two query tiles per CTA with P kept in TMEM;
    ``trace`` (int64 [4, 64, 4], two-tile only) receives SM-clock stamps of CTA 0's
    pipeline events (see csrc/attention.h).
    """
    T, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty(T, Hq * D, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(Hq, T, device=q.device, dtype=torch.float32)
    load().attention_fwd(q.contiguous(), k.contiguous(), v.contiguous(), o, lse, scale, status, bool(two_tile), trace)
    return o, lse


def attention_bwd(q, k, v, o, lse, dout, scale=None, status=None):
    """tcgen05 backward: (dq, dk, dv) shaped like (q, k, v)."""
    T, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dq, dk, dv = load().attention_bwd(q.contiguous(), k.contiguous(), v.contiguous(), o.contiguous(),
                                      dout.contiguous(), lse, scale, status)
    return dq, dk, dv


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = attention_fwd(q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        return attention_bwd(q, k, v, o, lse, do)


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Causal GQA attention on the tcgen05 kernels (T a multiple of 128, head_dim 128)."""
    return _FlashAttention.apply(q, k, v)


def causal_gqa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    T, Hq, D = q.shape
    qh = q.view(1, T, Hq, D).transpose(1, 2)
    kh = k.view(1, T, k.shape[1], D).transpose(1, 2)
    vh = v.view(1, T, v.shape[1], D).transpose(1, 2)
    o = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
    return o.transpose(1, 2).reshape(T, Hq * D)


def causal_gqa_attention_reference(q, k, v, return_lse=False):
    T, Hq, D = q.shape
    rep = Hq // k.shape[1]
    kk = k.float().repeat_interleave(rep, 1)
    vv = v.float().repeat_interleave(rep, 1)
    s = torch.einsum("thd,shd->hts", q.float(), kk) / D**0.5
    mask = torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.einsum("hts,shd->thd", s.softmax(-1), vv).reshape(T, Hq * D)
    if return_lse:
        return o, torch.logsumexp(s, -1)
    return o
