"""Language-model head + cross-entropy with a fused loss/gradient kernel.

The logits GEMM and both gradient GEMMs run on the tcgen05 GEMM (``spec_ep.ops.linear``;
the vocabulary's last 256-column tile is partial); the softmax cross-entropy and its
gradient run in one sm_100a kernel that overwrites the bf16 logits with
``(softmax - onehot) * scale`` so no fp32 copy of the [T, V] logits is ever stored.
"""
from __future__ import annotations

import torch

from ._ext import load
from .linear import dense_dgrad, dense_fwd, dense_wgrad


class _LMHeadXent(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, num_valid):
        C = load()
        logits = dense_fwd(h, w)  # [T, V] bf16
        loss = torch.empty(h.shape[0], device=h.device, dtype=torch.float32)
        if num_valid is not None:
            scale = 1.0 / max(int(num_valid), 1)
            C.xent_fwd_bwd(logits, labels, scale, loss)
            ctx.dev_scale = None
            out = loss.sum() * scale
        else:
            C.xent_fwd_bwd(logits, labels, 1.0, loss)
            valid = (labels >= 0).sum().clamp_min(1).float()
            ctx.dev_scale = 1.0 / valid
            out = loss.sum() / valid
        ctx.save_for_backward(h, w, logits)
        return out

    @staticmethod
    def backward(ctx, g):
        h, w, dlogits = ctx.saved_tensors
        dh = dense_dgrad(dlogits, w)
        dw = dense_wgrad(dlogits, h)
        s = g if ctx.dev_scale is None else g * ctx.dev_scale
        return dh * s.to(dh.dtype), dw * s.to(dw.dtype), None, None


def lm_head_xent(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, num_valid: int | None = None):
    """Mean next-token cross-entropy of ``h @ w.T`` against ``labels`` (int32, -1 = ignore).

    ``num_valid`` (labels >= 0, known on the host) lets the kernel apply the mean's
    scale directly; otherwise it is applied from a device-side count.
    """
    return _LMHeadXent.apply(h, w, labels.int().contiguous(), num_valid)


def lm_head_xent_reference(h, w, labels):
    logits = h.float() @ w.float().t()
    return torch.nn.functional.cross_entropy(logits, labels.long(), ignore_index=-1)
