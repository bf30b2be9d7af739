"""Fused per-head q/k RMSNorm + rotary embedding (Qwen3 attention pre-processing).

Input is the output of the fused QKV projection, ``[T, (Hq + 2*Hkv) * 128]``; the kernel
writes normalised+rotated ``q [T, Hq, 128]``, ``k [T, Hkv, 128]`` and copies ``v``.
Rotary convention is rotate-half (pairs ``(i, i + 64)``), as in transformers' Qwen3.
"""
from __future__ import annotations


import torch

from ._ext import load


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, wq, wk, Hq, Hkv, eps, theta, pos):
        C = load()
        T = qkv.shape[0]
        dev = qkv.device
        q = torch.empty(T, Hq, 128, device=dev, dtype=torch.bfloat16)
        k = torch.empty(T, Hkv, 128, device=dev, dtype=torch.bfloat16)
        v = torch.empty(T, Hkv, 128, device=dev, dtype=torch.bfloat16)
        rq = torch.empty(T, Hq, device=dev, dtype=torch.float32)
        rk = torch.empty(T, Hkv, device=dev, dtype=torch.float32)
        C.qk_norm_rope_fwd(qkv, wq, wk, q, k, v, rq, rk, pos, Hq, Hkv, eps, theta)
        ctx.save_for_backward(qkv, wq, wk, rq, rk, pos if pos is not None else torch.empty(0))
        ctx.cfg = (Hq, Hkv, theta, pos is not None)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, wq, wk, rq, rk, pos = ctx.saved_tensors
        Hq, Hkv, theta, has_pos = ctx.cfg
        C = load()
        dqkv = torch.empty_like(qkv)
        dwq = torch.zeros(128, device=qkv.device, dtype=torch.float32)
        dwk = torch.zeros(128, device=qkv.device, dtype=torch.float32)
        C.qk_norm_rope_bwd(qkv, wq, wk, rq, rk, dq.contiguous(), dk.contiguous(), dv.contiguous(), dqkv, dwq, dwk,
                           pos if has_pos else None, Hq, Hkv, theta)
        return dqkv, dwq.to(wq.dtype), dwk.to(wk.dtype), None, None, None, None, None


def qk_norm_rope(qkv, wq, wk, num_heads, num_kv_heads, eps=1e-6, theta=1e6, pos=None):
    return _QKNormRope.apply(qkv.contiguous(), wq, wk, num_heads, num_kv_heads, eps, theta, pos)


def qk_norm_rope_reference(qkv, wq, wk, Hq, Hkv, eps=1e-6, theta=1e6, pos=None):
    """fp32 PyTorch oracle: per-head RMSNorm then rotate-half RoPE."""
    T = qkv.shape[0]
    x = qkv.float().view(T, Hq + 2 * Hkv, 128)
    q, k, v = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]

    def norm(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w.float()

    q, k = norm(q, wq), norm(k, wk)
    p = (pos if pos is not None else torch.arange(T, device=qkv.device)).float()
    inv = theta ** (-torch.arange(0, 64, device=qkv.device).float() * 2 / 128)
    ang = p[:, None] * inv[None]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None]

    def rot(t):
        return torch.cat([-t[..., 64:], t[..., :64]], -1)

    return q * cos + rot(q) * sin, k * cos + rot(k) * sin, v
