"""Numerical self-check of the expert-parallel MoE layer on the ranks of a running job.

``ep_moe_check`` runs one small ``ep_moe`` forward + backward through the fused NVLink
kernels on every rank of the default process group and compares the output and every
gradient (tokens, gate weights, both expert weights) with a plain fp32 PyTorch MoE that
holds all experts. Each rank checks its own tokens; the expert-weight gradient of the
reference is summed over ranks (one all-reduce), since every rank's tokens reach every
expert. The result is the largest relative error over ranks, so a benchmark can print a
correctness figure next to each timed world size.

The reference computation mirrors the reference project's own oracle, an expert callback
applied to each routed copy and merged with its gate weight (src/rbd.py:485, :389-391).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


def moe_reference(x, te, tw, w_gu, w_d):
    """fp32 SwiGLU MoE: ``out[t] = sum_j tw[t, j] * FFN_{te[t, j]}(x[t])`` (all experts local)."""
    inter = w_d.shape[2]
    out = torch.zeros(x.shape, device=x.device, dtype=torch.float32)
    for j in range(te.shape[1]):
        for e in te[:, j].unique().tolist():
            m = te[:, j] == e
            gu = x[m] @ w_gu[e].t()
            out[m] += tw[m, j:j + 1] * ((F.silu(gu[:, :inter]) * gu[:, inter:]) @ w_d[e].t())
    return out


def _rel(a, b) -> float:
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


def ep_moe_check(device, T: int = 512, E: int = 16, k: int = 4, H: int = 512, inter: int = 256,
                 seed: int = 0) -> dict:
    """Max relative error of ``ep_moe`` vs the fp32 reference, max over ranks.

    Collective over the default group when it is initialised (every rank must call it);
    ``E`` must divide by the world size. Returns ``{"out", "dx", "dtopk_w", "dw_gu",
    "dw_d", "max"}``.
    """
    from ..parallel.ep import ExpertParallel, ep_moe

    dev = torch.device(device)
    ddp = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size() if ddp else 1
    rank = dist.get_rank() if ddp else 0
    g = torch.Generator().manual_seed(seed)
    w_gu_full = (torch.randn(E, 2 * inter, H, generator=g) / H**0.5).bfloat16().to(dev)
    w_d_full = (torch.randn(E, H, inter, generator=g) / inter**0.5).bfloat16().to(dev)
    epr = E // world
    w_gu = w_gu_full[rank * epr:(rank + 1) * epr].clone().requires_grad_()
    w_d = w_d_full[rank * epr:(rank + 1) * epr].clone().requires_grad_()
    gx = torch.Generator().manual_seed(seed * 7919 + 17 + rank)
    x = torch.randn(T, H, generator=gx).bfloat16().to(dev).requires_grad_()
    logits = torch.randn(T, E, generator=gx).to(dev)
    tw, te = torch.softmax(logits, -1).topk(k, -1)
    tw = (tw / tw.sum(-1, keepdim=True)).contiguous().requires_grad_()
    gout = torch.randn(T, H, generator=gx).bfloat16().to(dev)
    ep = ExpertParallel(E, k, H, max_tokens=T, device=dev)
    try:
        out = ep_moe(x, te.int(), tw, w_gu, w_d, ep)
        out.backward(gout)
        torch.cuda.synchronize(dev)
        ep.check()
        xr = x.detach().float().requires_grad_()
        twr = tw.detach().clone().requires_grad_()
        gur = w_gu_full.float().requires_grad_()
        dr = w_d_full.float().requires_grad_()
        ref = moe_reference(xr, te, twr, gur, dr)
        ref.backward(gout.float())
        dgu, dd = gur.grad, dr.grad
        if ddp:
            dist.all_reduce(dgu)
            dist.all_reduce(dd)
        errs = torch.tensor([_rel(out, ref), _rel(x.grad, xr.grad), _rel(tw.grad, twr.grad),
                             _rel(w_gu.grad, dgu[rank * epr:(rank + 1) * epr]),
                             _rel(w_d.grad, dd[rank * epr:(rank + 1) * epr])], device=dev, dtype=torch.float64)
        if ddp:
            dist.all_reduce(errs, op=dist.ReduceOp.MAX)
    finally:
        ep.close()
    names = ["out", "dx", "dtopk_w", "dw_gu", "dw_d"]
    res = {n: float(v) for n, v in zip(names, errs.tolist())}
    res["max"] = max(res.values())
    return res
