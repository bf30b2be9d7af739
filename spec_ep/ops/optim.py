"""Fused AdamW on the sm_100a kernel (csrc/elementwise.cu).

State precision per parameter:

* ``"fp32"``: fp32 master weights + fp32 moments (16 bytes/param with the bf16 weight).
* ``"8bit"``: block-wise 8-bit moments (Dettmers et al., ICLR 2022: int8 first moment and
  uint8 sqrt-second moment, one fp32 absmax scale per 32 values) and stochastic
  rounding of the bf16 weight (4.25 bytes/param with the bf16 weight). Used where fp32
  state does not fit, e.g. all 128 experts of a 30B-parameter MoE on one GPU.

Parameters may also be updated *inside the backward pass* through :meth:`apply_now`:
the MoE layer hands over each expert weight gradient as soon as its wgrad GEMM is done,
so no full-model gradient buffer ever exists (the gradient of one layer is transient),
or, through :meth:`fused_wgrad`, inside the weight-gradient GEMM itself: the tcgen05
kernel applies AdamW to each output tile in its epilogue and the gradient never reaches
HBM.
"""
from __future__ import annotations


import torch

from ._ext import load


class FusedAdamW:
    def __init__(self, params, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                 state_precision: str | dict = "fp32", max_grad_norm: float | None = None):
        self.params = [p for p in params]
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.step_count = 0
        self.max_grad_norm = max_grad_norm
        self.state: dict[int, dict] = {}
        self._precision = state_precision
        # stochastic-rounding seed of each parameter: its position in the optimizer
        self._seed = {id(p): i for i, p in enumerate(self.params)}
        for p in self.params:
            self._init_state(p)

    def precision_of(self, p) -> str:
        if isinstance(self._precision, dict):
            return self._precision.get(id(p), self._precision.get("default", "fp32"))
        return self._precision

    def _init_state(self, p):
        prec = getattr(p, "_sepx_state_precision", None) or self.precision_of(p)
        dev = p.device
        if prec == "fp32":
            st = dict(prec="fp32", master=p.detach().float().clone(),
                      m=torch.zeros(p.shape, device=dev, dtype=torch.float32),
                      v=torch.zeros(p.shape, device=dev, dtype=torch.float32))
        elif prec == "8bit":
            if p.numel() % 32:
                raise ValueError("8-bit optimizer state needs a multiple of 32 elements")
            nb = p.numel() // 32
            st = dict(prec="8bit",
                      mq=torch.zeros(p.numel(), device=dev, dtype=torch.int8),
                      ms=torch.zeros(nb, device=dev, dtype=torch.float32),
                      vq=torch.zeros(p.numel(), device=dev, dtype=torch.uint8),
                      vs=torch.zeros(nb, device=dev, dtype=torch.float32))
        else:
            raise ValueError(f"unknown optimizer state precision {prec!r}")
        self.state[id(p)] = st

    def state_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for st in self.state.values()
                   for t in st.values() if torch.is_tensor(t))

    # ---------------------------------------------------------------------------
    def _kernel_state(self, p):
        st = self.state[id(p)]
        if st["prec"] == "fp32":
            return 1, st["master"], st["m"], st["v"], None, None
        return 2, None, st["mq"], st["vq"], st["ms"], st["vs"]

    def _update(self, p, g, step, grad_scale=1.0):
        b1, b2 = self.betas
        kind, master, m, v, ms, vs = self._kernel_state(p)
        load().adamw_update(p.data, g.contiguous(), kind, master, m, v, ms, vs, self.lr, b1, b2, self.eps, self.wd,
                            step, grad_scale, self._seed[id(p)])

    def apply_now(self, p, grad):
        """Update ``p`` immediately with ``grad`` (optimizer-in-backward)."""
        self._update(p, grad, self.step_count + 1)

    def fused_wgrad(self, p, a, b, group_off, status=None):
        """``p[g] <- AdamW(p[g], a[rows_g]^T @ b[rows_g])`` in one tcgen05 GEMM (p is [G, M, N])."""
        b1, b2 = self.betas
        kind, master, m, v, ms, vs = self._kernel_state(p)
        load().gg_wgrad_adamw(a, b, group_off, p.data, kind, master, m, v, ms, vs, self.lr, b1, b2, self.eps,
                              self.wd, self.step_count + 1, 1.0, self._seed[id(p)], status)

    def step(self):
        """Update every parameter that has a ``.grad`` (those updated in backward have none)."""
        self.step_count += 1
        scale = 1.0
        if self.max_grad_norm is not None:
            grads = [p.grad for p in self.params if p.grad is not None]
            if grads:
                norm = torch.linalg.vector_norm(torch.stack([g.float().norm() for g in grads]))
                scale_t = (self.max_grad_norm / (norm + 1e-6)).clamp(max=1.0)
                for g in grads:
                    g.mul_(scale_t.to(g.dtype))
        for p in self.params:
            if p.grad is None:
                continue
            self._update(p, p.grad, self.step_count, scale)
            p.grad = None

    def zero_grad(self):
        for p in self.params:
            p.grad = None


def adamw_reference(p, g, m, v, lr, b1, b2, eps, wd, step):
    """fp32 PyTorch oracle of one AdamW step; returns (p, m, v)."""
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    mh = m / (1 - b1**step)
    vh = v / (1 - b2**step)
    p = p * (1 - lr * wd) - lr * mh / (vh.sqrt() + eps)
    return p, m, v


def encode_8bit(m: torch.Tensor, v: torch.Tensor):
    """fp32 moments -> the block-wise 8-bit codes the optimizer kernels read.

    Blocks are 32 consecutive values: ``mq = round(m * 127 / max|m|)`` (int8, nearest),
    ``vq = ceil(min(sqrt(v) * 255 / max sqrt(v), 255))`` (uint8, rounded up so a non-zero
    second moment never decodes to 0), ``ms = max|m|``, ``vs = max sqrt(v)`` per block.
    Returns ``(mq, ms, vq, vs)`` flattened; used to convert checkpointed state between
    precisions (the kernels themselves encode on the device).
    """
    m = m.float().reshape(-1, 32)
    sq = v.float().clamp_min(0).sqrt().reshape(-1, 32)
    ms = m.abs().amax(1)
    vs = sq.amax(1)
    em = torch.where(ms > 0, 127.0 / ms, torch.zeros_like(ms))
    ev = torch.where(vs > 0, 255.0 / vs, torch.zeros_like(vs))
    mq = torch.round(m * em[:, None]).clamp(-127, 127).to(torch.int8)
    vq = torch.ceil((sq * ev[:, None]).clamp(max=255.0)).to(torch.uint8)
    return mq.reshape(-1), ms, vq.reshape(-1), vs


def decode_8bit(mq: torch.Tensor, ms: torch.Tensor, vq: torch.Tensor, vs: torch.Tensor):
    """Block-wise 8-bit codes -> fp32 ``(m, v)`` (flattened), the inverse of :func:`encode_8bit`."""
    m = mq.reshape(-1, 32).float() * (ms.float() / 127.0)[:, None]
    s = vq.reshape(-1, 32).float() * (vs.float() / 255.0)[:, None]
    return m.reshape(-1), (s * s).reshape(-1)


def convert_state(src: dict, dst_prec: str, weight: torch.Tensor) -> dict:
    """One parameter's (or one expert's) optimizer state in another precision.

    ``src`` holds ``prec`` and the flat tensors of that precision (``master, m, v`` or
    ``mq, ms, vq, vs``); ``weight`` is the parameter's current (bf16) value, which becomes
    the fp32 master when 8-bit state (which keeps none) is widened. The conversion is
    lossy only where the narrower format is.
    """
    prec = src.get("prec", "fp32")
    if prec == dst_prec:
        return src
    if prec == "8bit" and dst_prec == "fp32":
        m, v = decode_8bit(src["mq"], src["ms"], src["vq"], src["vs"])
        return {"prec": "fp32", "master": weight.float().reshape(-1), "m": m, "v": v}
    if prec == "fp32" and dst_prec == "8bit":
        mq, ms, vq, vs = encode_8bit(src["m"], src["v"])
        return {"prec": "8bit", "mq": mq, "ms": ms, "vq": vq, "vs": vs}
    raise ValueError(f"cannot convert optimizer state {prec!r} -> {dst_prec!r}")


def bytes_per_param(precision: str) -> float:
    """Optimizer state bytes per parameter (excluding the bf16 weight itself)."""
    return {"fp32": 12.0, "8bit": 2.25}[precision]
