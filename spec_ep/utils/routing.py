"""Synthetic routing for benchmarks and tests.

Router logits are ``x @ W`` with ``W ~ N(0, 0.02)`` plus a per-expert bias chosen so
that expert popularity follows a Zipf law of exponent ``s``: expert of popularity rank
``r`` (1 = hottest, a random permutation of experts) gets bias ``-s * log(r)``, so its
softmax mass scales like ``r^-s`` on top of the data-dependent part.
"""
from __future__ import annotations

import torch


def zipf_bias(num_experts: int, s: float, seed: int = 0, device="cpu") -> torch.Tensor:
    g = torch.Generator().manual_seed(10_000 + seed)
    ranks = torch.randperm(num_experts, generator=g) + 1
    return (-s * torch.log(ranks.float())).to(device)


def synthetic_routing(T: int, hidden: int, num_experts: int, k: int, s: float = 1.0, seed: int = 0,
                      rank: int = 0, device="cpu", renorm: bool = True, bias_seed: int | None = None,
                      token_seed: int | None = None):
    """(x [T, H] bf16, topk_e [T, k] int32, topk_w [T, k] fp32) for one rank.

    ``seed`` selects the routing distribution (shared by all ranks); ``rank`` selects the
    rank's tokens. Computed with plain torch so every implementation sees the same routes.
    ``bias_seed`` (default ``seed``) draws the popularity order alone, with the router
    weights kept: a new ``bias_seed`` moves which experts are hot (drifting popularity);
    ``token_seed`` (default ``seed``) draws the tokens alone.
    """
    g = torch.Generator().manual_seed((seed if token_seed is None else token_seed) * 1000 + rank)
    x = torch.randn(T, hidden, generator=g)
    gw = torch.Generator().manual_seed(seed)
    w = torch.randn(hidden, num_experts, generator=gw) * 0.02
    logits = x @ w + zipf_bias(num_experts, s, seed if bias_seed is None else bias_seed)
    p = torch.softmax(logits, -1)
    topk_w, topk_e = p.topk(k, -1)
    if renorm:
        topk_w = topk_w / topk_w.sum(-1, keepdim=True)
    return x.to(device, torch.bfloat16), topk_e.int().to(device), topk_w.float().to(device)


def dedup_bound_rows(topk_e: torch.Tensor, experts_per_rank: int, rank: int, world: int) -> dict:
    """Rows per token that cross to other ranks: naive (per copy) vs per-rank dedup."""
    dst = torch.div(topk_e.long(), experts_per_rank, rounding_mode="floor")
    T = topk_e.shape[0]
    naive = (dst != rank).sum().item() / T
    hot = torch.zeros(T, world, dtype=torch.bool)
    hot.scatter_(1, dst.cpu(), True)
    dedup = (hot.sum().item() - hot[:, rank].sum().item()) / T
    return {"naive_rows_per_token": naive, "dedup_rows_per_token": dedup}
