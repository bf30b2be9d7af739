"""Fused expert-parallel MoE layer (dispatch -> tcgen05 GEMMs -> combine) on one GPU,
forward and backward, against an fp32 PyTorch reference of the same SwiGLU MoE."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _moe_reference(x, topk_e, topk_w, w_gu, w_d):
    xf = x.float()
    out = torch.zeros_like(xf)
    I = w_d.shape[2]
    for j in range(topk_e.shape[1]):
        for e in topk_e[:, j].unique().tolist():
            m = topk_e[:, j] == e
            gu = xf[m] @ w_gu[e].float().t()
            h = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
            out[m] += topk_w[m, j:j + 1] * (h @ w_d[e].float().t())
    return out


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("T,E,k,H,I", [(512, 8, 2, 256, 256), (1024, 16, 4, 512, 256), (777, 32, 8, 256, 512)])
def test_ep_moe_single_gpu_forward_backward(T, E, k, H, I):
    from spec_ep.parallel.ep import ExpertParallel, ep_moe

    torch.manual_seed(0)
    dev = "cuda"
    x = torch.randn(T, H, device=dev).bfloat16().requires_grad_()
    logits = torch.randn(T, E, device=dev)
    p = torch.softmax(logits, -1)
    topk_w, topk_e = p.topk(k, -1)
    topk_w = (topk_w / topk_w.sum(-1, keepdim=True)).requires_grad_()
    w_gu = (torch.randn(E, 2 * I, H, device=dev) / H**0.5).bfloat16().requires_grad_()
    w_d = (torch.randn(E, H, I, device=dev) / I**0.5).bfloat16().requires_grad_()
    ep = ExpertParallel(E, k, H, max_tokens=1024)
    out = ep_moe(x, topk_e.int(), topk_w, w_gu, w_d, ep)
    g = torch.randn_like(out)
    out.backward(g)
    torch.cuda.synchronize()
    ep.check()

    xr = x.detach().float().requires_grad_()
    wr = topk_w.detach().clone().requires_grad_()
    gur = w_gu.detach().float().requires_grad_()
    dr = w_d.detach().float().requires_grad_()
    ref = _moe_reference(xr, topk_e, wr, gur, dr)
    ref.backward(g.float())
    assert _rel(out, ref) < 2e-2
    assert _rel(x.grad, xr.grad) < 3e-2
    assert _rel(topk_w.grad, wr.grad) < 3e-2
    assert _rel(w_gu.grad, gur.grad) < 3e-2
    assert _rel(w_d.grad, dr.grad) < 3e-2
    ep.close()


def test_ep_moe_deterministic_and_repeatable():
    from spec_ep.parallel.ep import ExpertParallel, ep_moe

    torch.manual_seed(1)
    T, E, k, H, I = 1024, 16, 4, 256, 256
    x = torch.randn(T, H, device="cuda").bfloat16()
    topk_e = torch.rand(T, E, device="cuda").topk(k, -1).indices.int()
    topk_w = torch.rand(T, k, device="cuda")
    w_gu = (torch.randn(E, 2 * I, H, device="cuda") / 16).bfloat16()
    w_d = (torch.randn(E, H, I, device="cuda") / 16).bfloat16()
    ep = ExpertParallel(E, k, H, max_tokens=T)
    a = ep_moe(x, topk_e, topk_w, w_gu, w_d, ep)
    b = ep_moe(x, topk_e, topk_w, w_gu, w_d, ep)
    torch.cuda.synchronize()
    ep.check()
    assert torch.equal(a, b)
    ep.close()


@pytest.mark.gpu
def test_ep_layers_replayed_as_cuda_graph_match_eager():
    """Two expert-parallel inference layers (dispatch, SwiGLU expert GEMMs, combine) captured
    once and replayed on fresh inputs give the eager results bit for bit."""
    from spec_ep.ops.grouped_gemm import gg_fwd, gg_swiglu_fwd
    from spec_ep.parallel.ep import EPGraph, ExpertParallel

    torch.manual_seed(3)
    E, k, H, I, T = 16, 4, 256, 128, 128
    w_gu = (torch.randn(E, 2 * I, H, device="cuda") / H**0.5).bfloat16()
    w_d = (torch.randn(E, H, I, device="cuda") / I**0.5).bfloat16()

    def layers(ep, x, te, tw, static):
        for _ in range(2):
            st = ep.dispatch_fwd(x, te, tw, static_rows=static)
            h, _ = gg_swiglu_fwd(st.xp, w_gu, st.group_off, status=ep.status)
            y = gg_fwd(h, w_d, st.group_off, status=ep.status)
            x = ep.combine_fwd(y, st)
        return x

    def inputs(seed):
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        te = torch.stack([torch.randperm(E, device="cuda", generator=g)[:k] for _ in range(T)]).int()
        tw = torch.rand(T, k, device="cuda", generator=g)
        return x, te, tw

    eager_ep = ExpertParallel(E, k, H, max_tokens=T)
    graph_ep = ExpertParallel(E, k, H, max_tokens=T)
    xs, tes, tws = inputs(0)
    graph = EPGraph(graph_ep, lambda: layers(graph_ep, xs, tes, tws, True))
    for seed in (1, 2, 3):
        x, te, tw = inputs(seed)
        xs.copy_(x)
        tes.copy_(te)
        tws.copy_(tw)
        got = graph.replay().clone()
        want = layers(eager_ep, x, te, tw, False)
        torch.cuda.synchronize()
        assert torch.equal(got, want), seed
    graph_ep.check()
    eager_ep.check()
    del graph
    graph_ep.close()
    eager_ep.close()


def test_row_budget_pass_matches_exact_sizes_and_recovers_from_overflow():
    """Inside begin_pass / end_pass the receive buffers come from learned row budgets
    (no device->host read per layer). The result equals the exact-size path bit for bit;
    a budget that is too small empties the layer, raises the miss flag, and the pass
    run again with the grown budget gives the exact result."""
    from spec_ep.parallel.ep import ExpertParallel, ep_moe

    torch.manual_seed(1)
    T, E, k, H, I = 512, 16, 4, 256, 256
    x = torch.randn(T, H, device="cuda").bfloat16()
    p = torch.softmax(torch.randn(T, E, device="cuda"), -1)
    tw, te = p.topk(k, -1)
    tw = tw / tw.sum(-1, keepdim=True)
    w_gu = (torch.randn(E, 2 * I, H, device="cuda") / H**0.5).bfloat16()
    w_d = (torch.randn(E, H, I, device="cuda") / I**0.5).bfloat16()
    ep = ExpertParallel(E, k, H, max_tokens=T)

    def layers():  # two layer calls per pass
        y = ep_moe(x, te.int(), tw, w_gu, w_d, ep)
        return ep_moe(y, te.int(), tw, w_gu, w_d, ep)

    exact = layers()  # outside a pass: exact sizes
    ep.begin_pass()
    learn = layers()  # first pass: learns the budgets (exact sizes)
    assert not ep.end_pass()
    assert ep._budget >= T * k
    ep.begin_pass()
    budgeted = layers()  # no host read between the layers
    assert not ep.end_pass()
    assert torch.equal(learn, exact) and torch.equal(budgeted, exact)
    ep._budget = 64  # far too small: the first call overflows
    ep.begin_pass()
    layers()
    assert ep.end_pass()  # reported, and the budget grown
    assert ep._budget >= T * k
    ep.begin_pass()
    again = layers()
    assert not ep.end_pass()
    torch.cuda.synchronize()
    ep.check()  # an overflowed budget is not an error
    assert torch.equal(again, exact)
    ep.close()
