"""Dense projections on the tcgen05 GEMM (``spec_ep.ops.linear``) against fp32 PyTorch:
forward, input gradient and weight gradient, at the model's projection shapes (fused
QKV, attention output, router with 128 outputs, and a vocabulary whose last 256-column
tile is partial), plus small routers and token counts that take the zero-padded path;
(4096, 2048, 128) and (4160, 512, 8) take the weight gradient split over token ranges."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("T,K,N", [(512, 512, 1280), (512, 1024, 512), (256, 512, 128), (256, 512, 4224),
                                   (384, 256, 256), (256, 512, 8), (200, 512, 48), (4096, 2048, 128),
                                   (4160, 512, 8)])
def test_linear_forward_backward_matches_fp32(T, K, N):
    from spec_ep.ops.linear import linear

    torch.manual_seed(0)
    x = torch.randn(T, K, device="cuda").bfloat16().requires_grad_()
    w = (torch.randn(N, K, device="cuda") / K**0.5).bfloat16().requires_grad_()
    y = linear(x, w)
    g = torch.randn(T, N, device="cuda").bfloat16()
    y.backward(g)
    torch.cuda.synchronize()
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = xr @ wr.t()
    yr.backward(g.float())
    assert y.shape == (T, N) and y.dtype == torch.bfloat16
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-2



def test_lm_head_xent_on_own_gemm_matches_reference():
    from spec_ep.ops.loss import lm_head_xent, lm_head_xent_reference

    torch.manual_seed(1)
    T, H, V = 256, 512, 4224
    h = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    w = (torch.randn(V, H, device="cuda") * 0.05).bfloat16().requires_grad_()
    labels = torch.randint(0, V, (T,), device="cuda").int()
    labels[-1] = -1
    loss = lm_head_xent(h, w, labels, T - 1)
    loss.backward()
    hr = h.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    ref = lm_head_xent_reference(hr, wr, labels)
    ref.backward()
    assert abs(loss.item() - ref.item()) < 2e-2 * abs(ref.item())
    assert _rel(h.grad, hr.grad) < 3e-2
    assert _rel(w.grad, wr.grad) < 3e-2


@pytest.mark.parametrize("bias", [False, True])
def test_router_front_matches_projection_then_router(bias):
    """One launch (router GEMM whose epilogue does softmax / top-k / renormalisation and the
    routing tables) against the projection followed by the standalone router kernel and
    the table lookup: same experts, weights and gradients to fp32 rounding."""
    from spec_ep.ops.linear import linear
    from spec_ep.ops.router import router_front, router_topk

    torch.manual_seed(4)
    T, H, E, k = 1000, 2048, 128, 8
    h = torch.randn(T, H, device="cuda").bfloat16()
    w = (torch.randn(E, H, device="cuda") / H**0.5).bfloat16()
    sel = (0.01 * torch.rand(E, device="cuda")) if bias else None
    lgb = (0.5 * torch.randn(E, device="cuda")) if bias else None
    e2r = (torch.arange(E, device="cuda") // 16).int()
    e2l = (torch.arange(E, device="cuda") % 16).int()
    g = torch.randn(T, k, device="cuda")

    h1, w1 = h.clone().requires_grad_(), w.clone().requires_grad_()
    tw1, te1, dst, meta = router_front(h1, w1, k, True, sel, lgb, (e2r, e2l))
    (tw1 * g).sum().backward()

    h2, w2 = h.clone().requires_grad_(), w.clone().requires_grad_()
    logits = linear(h2, w2).float()
    if lgb is not None:
        logits = logits + lgb
    tw2, te2 = router_topk(logits, k, True, sel)
    (tw2 * g).sum().backward()
    torch.cuda.synchronize()

    same = (te1 == te2).all(1)
    assert same.float().mean().item() > 0.995  # near-ties may order differently
    assert torch.equal(dst[same], e2r[te1[same].long()]) and torch.equal(meta[same], e2l[te1[same].long()])
    assert (tw1[same] - tw2[same]).abs().max().item() < 1e-5
    assert _rel(h1.grad[same], h2.grad[same]) < 2e-2 and _rel(w1.grad, w2.grad) < 2e-2

