"""tcgen05 causal GQA attention against an fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("two_tile", [False, True])
@pytest.mark.parametrize("T,Hq,Hkv", [(128, 2, 1), (512, 4, 2), (1024, 8, 1), (384, 4, 4)])
def test_attention_fwd(T, Hq, Hkv, two_tile):
    from spec_ep.ops.attention import attention_fwd, causal_gqa_attention_reference

    torch.manual_seed(0)
    q = torch.randn(T, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, lse = attention_fwd(q, k, v, status=st, two_tile=two_tile)
    torch.cuda.synchronize()
    assert st.item() == 0
    ref, ref_lse = causal_gqa_attention_reference(q, k, v, return_lse=True)
    assert _rel(o, ref) < 2e-2
    assert (lse - ref_lse).abs().max().item() < 2e-2


@pytest.mark.parametrize("two_tile", [False, True])
def test_attention_fwd_large_logits_lazy_rescale(two_tile):
    """Rows whose max keeps growing across key blocks exercise the O rescaling path."""
    from spec_ep.ops.attention import attention_fwd, causal_gqa_attention_reference

    torch.manual_seed(1)
    T = 1024
    q = (torch.randn(T, 2, 128, device="cuda") * 3).bfloat16()
    k = (torch.randn(T, 1, 128, device="cuda") * 3).bfloat16()
    k += torch.linspace(0, 4, T, device="cuda").view(T, 1, 1).bfloat16()  # later keys score higher
    v = torch.randn(T, 1, 128, device="cuda").bfloat16()
    o, lse = attention_fwd(q, k, v, two_tile=two_tile)
    ref, ref_lse = causal_gqa_attention_reference(q, k, v, return_lse=True)
    torch.cuda.synchronize()
    assert _rel(o, ref) < 3e-2
    assert ((lse - ref_lse).abs() / ref_lse.abs().clamp_min(1)).max().item() < 1e-2


@pytest.mark.parametrize("T,Hq,Hkv", [(128, 2, 1), (512, 4, 2), (768, 8, 1)])
def test_attention_bwd(T, Hq, Hkv):
    from spec_ep.ops.attention import causal_gqa_attention_reference, flash_attention

    torch.manual_seed(2)
    q = torch.randn(T, Hq, 128, device="cuda").bfloat16().requires_grad_()
    k = torch.randn(T, Hkv, 128, device="cuda").bfloat16().requires_grad_()
    v = torch.randn(T, Hkv, 128, device="cuda").bfloat16().requires_grad_()
    do = torch.randn(T, Hq * 128, device="cuda").bfloat16()
    o = flash_attention(q, k, v)
    o.backward(do)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = causal_gqa_attention_reference(qf, kf, vf)
    ref.backward(do.float())
    assert _rel(o, ref) < 2e-2
    for got, want in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        assert got.shape == want.shape
        assert _rel(got, want) < 3e-2
