"""Dense projections on the tcgen05 GEMM (csrc/grouped_gemm.cu, one group).

``linear(x, w)`` is ``x @ w.T`` with autograd, for the model's dense layers (fused QKV,
attention output, router, LM head): forward and input gradient run as one-group ragged-M
GEMMs (256-column tiles on CTA pairs, a partial last tile clipped by the TMA stores), the
weight gradient as a one-group ragged-K GEMM with a bf16 epilogue. Shapes: the reduction
dimension a multiple of 64, output columns a multiple of 32 (128 for the weight gradient's
rows), token count a multiple of 64 for the weight gradient.

Reference parity: the reference's dense GEMM is ``torch.mm`` (benchmark/compute.py:57-62)
and its model's projections are transformers ``nn.Linear`` layers (scripts/ds_moe.py:26-48).
"""
from __future__ import annotations

import torch

from ._ext import load

_OFFSETS: dict = {}


def _rows_offsets(rows: int, device) -> torch.Tensor:
    """Cached device tensor [0, rows] (the single group of a dense GEMM)."""
    key = (rows, str(device))
    t = _OFFSETS.get(key)
    if t is None:
        t = torch.tensor([0, rows], dtype=torch.int32, device=device)
        _OFFSETS[key] = t
    return t


def _pad0(t: torch.Tensor, mult: int) -> torch.Tensor:
    """``t`` with zero rows appended up to a multiple of ``mult`` rows."""
    r = (-t.shape[0]) % mult
    return t if r == 0 else torch.cat([t, t.new_zeros((r,) + tuple(t.shape[1:]))])


def _pad1(t: torch.Tensor, mult: int) -> torch.Tensor:
    """``t`` with zero columns appended up to a multiple of ``mult`` columns."""
    r = (-t.shape[1]) % mult
    return t if r == 0 else torch.nn.functional.pad(t, (0, r))


def dense_fwd(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x [T, K] @ w[N, K].T -> [T, N]`` (bf16). Output widths the kernel does not tile
    (N below 256 and not a multiple of 128, or not a multiple of 32) run on weights padded
    with zero rows; the model shapes need no padding."""
    x = x.contiguous()
    N = w.shape[0]
    wp = w if (N % 128 == 0 or (N > 256 and N % 32 == 0)) else _pad0(w, 128)
    out = torch.empty(x.shape[0], wp.shape[0], device=x.device, dtype=torch.bfloat16)
    load().gg_fwd(x, wp.contiguous().unsqueeze(0), _rows_offsets(x.shape[0], x.device), out, None)
    return out if wp is w else out[:, :N].contiguous()


def dense_dgrad(gy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``gy [T, N] @ w [N, K] -> [T, K]`` (input gradient of ``x @ w.T``). The reduction
    over N runs in 64-wide steps: other N are padded with zeros."""
    gy = _pad1(gy.contiguous(), 64).contiguous()
    wp = _pad0(w, 64).contiguous()
    out = torch.empty(gy.shape[0], w.shape[1], device=gy.device, dtype=torch.bfloat16)
    load().gg_dgrad(gy, wp.unsqueeze(0), _rows_offsets(gy.shape[0], gy.device), out, None)
    return out


_SM_COUNT: dict = {}


def _sm_count(device) -> int:
    key = str(device)
    if key not in _SM_COUNT:
        _SM_COUNT[key] = torch.cuda.get_device_properties(device).multi_processor_count
    return _SM_COUNT[key]


def _split_offsets(rows: int, parts: int, device) -> torch.Tensor:
    """Cached device tensor of ``parts`` equal row ranges of ``rows`` (multiples of 64)."""
    key = ("split", rows, parts, str(device))
    t = _OFFSETS.get(key)
    if t is None:
        step = rows // parts
        t = torch.tensor([i * step for i in range(parts)] + [rows], dtype=torch.int32, device=device)
        _OFFSETS[key] = t
    return t


def wgrad_split(N: int, K: int, T: int, sms: int) -> int:
    """Reduction splits for a weight gradient with an ``N x K`` output over ``T`` tokens:
    1 when its 128 x 256 output tiles already fill half the SMs, else enough equal token
    ranges (of at least 256 rows, each a multiple of 64) to give about one tile per SM."""
    tiles = -(-N // 128) * -(-K // 256)
    if 2 * tiles >= sms or T < 512:
        return 1
    parts = min(T // 256, -(-sms // tiles))
    while parts > 1 and (T % parts or (T // parts) % 64):
        parts -= 1
    return max(parts, 1)


def dense_wgrad(gy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """``gy [T, N].T @ x [T, K] -> [N, K]`` (weight gradient of ``x @ w.T``, bf16). Rows of
    the output come in 128-row tiles and tokens in 64-row steps: others are zero-padded.

    An output too small to fill the GPU (the router's 128 x 2048: 8 tiles) splits the
    token dimension: each token range is one group of the ragged-K GEMM writing an fp32
    partial, and the partials are summed in fp32 before the one rounding to bf16."""
    N, T = gy.shape[1], gy.shape[0]
    gyp = _pad0(_pad1(gy.contiguous(), 128), 64).contiguous()
    xp = _pad0(x.contiguous(), 64).contiguous()
    parts = wgrad_split(gyp.shape[1], x.shape[1], xp.shape[0], _sm_count(x.device))
    if parts > 1:
        part = torch.empty(parts, gyp.shape[1], x.shape[1], device=x.device, dtype=torch.float32)
        load().gg_wgrad(gyp, xp, _split_offsets(xp.shape[0], parts, x.device), part, None)
        out = part.sum(0).to(torch.bfloat16)
    else:
        out = torch.empty(gyp.shape[1], x.shape[1], device=x.device, dtype=torch.bfloat16)
        load().gemm_wgrad_bf16(gyp, xp, _rows_offsets(xp.shape[0], x.device), out, None)
    return out if gyp.shape[1] == N else out[:N]


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return dense_fwd(x, w)

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gx = dense_dgrad(gy, w) if ctx.needs_input_grad[0] else None
        gw = dense_wgrad(gy, x) if ctx.needs_input_grad[1] else None
        return gx, gw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` for 2-D bf16 ``x [T, K]`` and ``w [N, K]`` on the tcgen05 GEMM."""
    return _Linear.apply(x, w)


def linear_reference(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return x.float() @ w.float().t()
