"""Python wrappers for the tcgen05 grouped GEMM (csrc/grouped_gemm.cu).

Row groups are described by ``group_off`` (int32, G+1 entries, on the device): group g
owns rows ``[group_off[g], group_off[g+1])`` of the row-major activations. Offsets
never need to reach the host, so a full MoE layer runs without a device sync.

Weight layouts follow transformers' Qwen3-MoE experts (``gate_up_proj [E, 2I, H]``,
``down_proj [E, H, I]``), so checkpoints load without reshuffling.
"""
from __future__ import annotations

import torch

from ._ext import load


def gg_fwd(a, w, group_off, out=None, status=None):
    """out[r] = a[r] @ w[g].T for r in group g.  a [R, K], w [G, N, K] -> [R, N] (bf16)."""
    if out is None:
        out = torch.empty(a.shape[0], w.shape[1], device=a.device, dtype=torch.bfloat16)
    load().gg_fwd(a, w, group_off, out, status)
    return out


def gg_dgrad(a, w, group_off, out=None, status=None):
    """out[r] = a[r] @ w[g] for r in group g.  a [R, K], w [G, K, N] -> [R, N] (bf16)."""
    if out is None:
        out = torch.empty(a.shape[0], w.shape[2], device=a.device, dtype=torch.bfloat16)
    load().gg_dgrad(a, w, group_off, out, status)
    return out


def gg_swiglu_fwd(a, w_gu, group_off, h=None, gu=None, status=None):
    """[g|u] = a @ w_gu[g].T; returns h = silu(g)*u [R, I] and gu [R, 2I]."""
    R, I2 = a.shape[0], w_gu.shape[1]
    if h is None:
        h = torch.empty(R, I2 // 2, device=a.device, dtype=torch.bfloat16)
    if gu is None:
        gu = torch.empty(R, I2, device=a.device, dtype=torch.bfloat16)
    load().gg_swiglu_fwd(a, w_gu, group_off, h, gu, status)
    return h, gu


def gg_swiglu_bwd(dy, w_down, group_off, gu, row_w, dgu=None, hw=None, row_dw=None, status=None):
    """Backward through ``y = w_row * (silu(g)*u) @ w_down[g].T`` for unweighted dy rows.

    Returns (dgu [R, 2I], hw = w_row*h [R, I], row_dw [R] += <dy @ w_down[g], h>).
    """
    R, I = dy.shape[0], w_down.shape[2]
    if dgu is None:
        dgu = torch.empty(R, 2 * I, device=dy.device, dtype=torch.bfloat16)
    if hw is None:
        hw = torch.empty(R, I, device=dy.device, dtype=torch.bfloat16)
    if row_dw is None:
        row_dw = torch.zeros(R, device=dy.device, dtype=torch.float32)
    load().gg_swiglu_bwd(dy, w_down, group_off, gu, row_w, dgu, hw, row_dw, status)
    return dgu, hw, row_dw


def gg_wgrad(a, b, group_off, G, out=None, status=None):
    """out[g] = a[rows_g].T @ b[rows_g] in fp32.  a [R, M], b [R, N] -> [G, M, N].

    Group offsets must be multiples of 64 and rows between groups must be zero-filled.
    """
    if out is None:
        out = torch.empty(G, a.shape[1], b.shape[1], device=a.device, dtype=torch.float32)
    load().gg_wgrad(a, b, group_off, out, status)
    return out
