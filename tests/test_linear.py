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
