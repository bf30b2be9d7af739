"""RMSNorm on the sm_100a kernel (csrc/elementwise.cu), with autograd.

Besides the plain ``rms_norm``, two forms for a pre-norm residual stream, which fold the
stream's bf16 add and the sum of its gradients into the norm kernels (same bits as
writing them out as separate tensor ops):

* ``rms_norm_res(x, w)`` -> ``(rms_norm(x, w), x)``: the second output carries ``x`` on to
  the residual add, and the backward adds its gradient into the norm's input gradient.
* ``add_rms_norm(x, o, w)`` -> ``(s, rms_norm(s, w))`` with ``s = x + o``: the residual
  add and the next norm in one kernel; the backward adds the gradient that reaches ``s``
  from its other uses into the norm's input gradient and returns it for both ``x`` and
  ``o``.
"""
from __future__ import annotations

import torch

from ._ext import load


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        C = load()
        xc = x.contiguous()
        y = torch.empty_like(xc)
        rstd = torch.empty(xc.numel() // xc.shape[-1], device=x.device, dtype=torch.float32)
        C.rmsnorm_fwd(xc, w, y, rstd, eps, None, None)
        ctx.save_for_backward(xc, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        C = load()
        dx = torch.empty_like(x)
        dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        C.rmsnorm_bwd(x, w, rstd, dy.contiguous(), dx, dw, None)
        return dx, dw.to(w.dtype), None


class _RMSNormRes(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        C = load()
        xc = x.contiguous()
        y = torch.empty_like(xc)
        rstd = torch.empty(xc.numel() // xc.shape[-1], device=x.device, dtype=torch.float32)
        C.rmsnorm_fwd(xc, w, y, rstd, eps, None, None)
        ctx.save_for_backward(xc, w, rstd)
        return y, xc.view_as(xc)

    @staticmethod
    def backward(ctx, dy, dres):
        x, w, rstd = ctx.saved_tensors
        C = load()
        dx = torch.empty_like(x)
        dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        if dy is None:
            dy = torch.zeros_like(x)
        C.rmsnorm_bwd(x, w, rstd, dy.contiguous(), dx, dw, None if dres is None else dres.contiguous())
        return dx, dw.to(w.dtype), None


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, o, w, eps):
        C = load()
        xc, oc = x.contiguous(), o.contiguous()
        s = torch.empty_like(xc)
        y = torch.empty_like(xc)
        rstd = torch.empty(xc.numel() // xc.shape[-1], device=x.device, dtype=torch.float32)
        C.rmsnorm_fwd(xc, w, y, rstd, eps, oc, s)
        ctx.save_for_backward(s, w, rstd)
        return s, y

    @staticmethod
    def backward(ctx, ds, dy):
        s, w, rstd = ctx.saved_tensors
        C = load()
        dx = torch.empty_like(s)
        dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        if dy is None:
            dy = torch.zeros_like(s)
        C.rmsnorm_bwd(s, w, rstd, dy.contiguous(), dx, dw, None if ds is None else ds.contiguous())
        return dx, dx, dw.to(w.dtype), None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = weight * x / sqrt(mean(x^2) + eps) over the last dimension (bf16 in/out)."""
    return _RMSNorm.apply(x, weight, eps)


def rms_norm_res(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """``(rms_norm(x, weight), x)``: the second output is ``x`` for the residual path, whose
    gradient the norm's backward adds into its own input gradient (one kernel)."""
    return _RMSNormRes.apply(x, weight, eps)


def add_rms_norm(x: torch.Tensor, o: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """``(s, rms_norm(s, weight))`` with ``s = x + o`` (bf16), in one kernel each way."""
    return _AddRMSNorm.apply(x, o, weight, eps)


def rms_norm_reference(x, weight, eps=1e-6):
    """fp32 PyTorch oracle."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float())
