"""The fp32 MoE oracle of the EP self-check (runs on CPU): equal to a per-token loop, and
differentiable in every input it is compared on."""
import torch
import torch.nn.functional as F

from spec_ep.utils.selfcheck import moe_reference


def _per_token(x, te, tw, w_gu, w_d):
    inter = w_d.shape[2]
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(te.shape[1]):
            e = int(te[t, j])
            gu = x[t] @ w_gu[e].t()
            out[t] += tw[t, j] * ((F.silu(gu[:inter]) * gu[inter:]) @ w_d[e].t())
    return out


def test_moe_reference_matches_a_per_token_loop():
    torch.manual_seed(0)
    T, E, k, H, inter = 37, 6, 3, 16, 8
    x = torch.randn(T, H)
    w_gu = torch.randn(E, 2 * inter, H) / H**0.5
    w_d = torch.randn(E, H, inter) / inter**0.5
    tw, te = torch.softmax(torch.randn(T, E), -1).topk(k, -1)
    got = moe_reference(x, te, tw, w_gu, w_d)
    want = _per_token(x, te, tw, w_gu, w_d)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)


def test_moe_reference_gradients_flow():
    torch.manual_seed(1)
    T, E, k, H, inter = 20, 4, 2, 8, 4
    x = torch.randn(T, H, requires_grad=True)
    w_gu = (torch.randn(E, 2 * inter, H) / H**0.5).requires_grad_()
    w_d = (torch.randn(E, H, inter) / inter**0.5).requires_grad_()
    tw, te = torch.softmax(torch.randn(T, E), -1).topk(k, -1)
    tw = tw.detach().requires_grad_()
    moe_reference(x, te, tw, w_gu, w_d).sum().backward()
    for t in (x, tw, w_gu, w_d):
        assert t.grad is not None and torch.isfinite(t.grad).all() and t.grad.abs().sum() > 0
