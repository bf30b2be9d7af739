"""Causal grouped-query attention.

q [T, Hq, D], k/v [T, Hkv, D] (token-major, as written by the fused q/k-norm+RoPE
kernel) -> out [T, Hq * D]. Runs torch's scaled_dot_product_attention with GQA.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_gqa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    T, Hq, D = q.shape
    qh = q.view(1, T, Hq, D).transpose(1, 2)
    kh = k.view(1, T, k.shape[1], D).transpose(1, 2)
    vh = v.view(1, T, v.shape[1], D).transpose(1, 2)
    o = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
    return o.transpose(1, 2).reshape(T, Hq * D)


def causal_gqa_attention_reference(q, k, v):
    T, Hq, D = q.shape
    rep = Hq // k.shape[1]
    kk = k.float().repeat_interleave(rep, 1)
    vv = v.float().repeat_interleave(rep, 1)
    s = torch.einsum("thd,shd->hts", q.float(), kk) / D**0.5
    mask = torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    return torch.einsum("hts,shd->thd", s.softmax(-1), vv).reshape(T, Hq * D)
