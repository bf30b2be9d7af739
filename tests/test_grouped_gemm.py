"""Numerics of the tcgen05 grouped GEMM against a plain fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _offsets(sizes, align=1):
    off = [0]
    for s in sizes:
        off.append(off[-1] + ((s + align - 1) // align) * align)
    return off


def _rel_err(out, ref):
    return ((out.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


def _status():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("N", [256, 384])
def test_fwd_ragged_m(N):
    from spec_ep.ops.grouped_gemm import gg_fwd

    torch.manual_seed(0)
    sizes = [100, 0, 300, 37, 128]
    off = _offsets(sizes)
    R, K, G = off[-1], 256, len(sizes)
    a = torch.randn(R, K, device="cuda").bfloat16()
    w = (torch.randn(G, N, K, device="cuda") / K**0.5).bfloat16()
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    st = _status()
    out = gg_fwd(a, w, go, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    ref = torch.cat([a[off[g]:off[g + 1]].float() @ w[g].float().T for g in range(G)])
    assert _rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("N", [256, 128])
def test_dgrad_ragged_m(N):
    from spec_ep.ops.grouped_gemm import gg_dgrad

    torch.manual_seed(1)
    sizes = [64, 200, 5, 0, 129]
    off = _offsets(sizes)
    R, K, G = off[-1], 384, len(sizes)
    a = torch.randn(R, K, device="cuda").bfloat16()
    w = (torch.randn(G, K, N, device="cuda") / K**0.5).bfloat16()
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    st = _status()
    out = gg_dgrad(a, w, go, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    ref = torch.cat([a[off[g]:off[g + 1]].float() @ w[g].float() for g in range(G)])
    assert _rel_err(out, ref) < 1e-2


def test_swiglu_fwd():
    from spec_ep.ops.grouped_gemm import gg_swiglu_fwd

    torch.manual_seed(2)
    sizes = [130, 64, 0, 250]
    off = _offsets(sizes)
    R, K, G, I = off[-1], 256, len(sizes), 256
    a = torch.randn(R, K, device="cuda").bfloat16()
    w = (torch.randn(G, 2 * I, K, device="cuda") / K**0.5).bfloat16()
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    st = _status()
    h, gu = gg_swiglu_fwd(a, w, go, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    gu_ref = torch.cat([a[off[g]:off[g + 1]].float() @ w[g].float().T for g in range(G)])
    g_, u_ = gu_ref[:, :I], gu_ref[:, I:]
    h_ref = torch.nn.functional.silu(g_) * u_
    assert _rel_err(gu, gu_ref) < 1e-2
    assert _rel_err(h, h_ref) < 2e-2


def test_swiglu_bwd():
    from spec_ep.ops.grouped_gemm import gg_swiglu_bwd

    torch.manual_seed(3)
    sizes = [128, 70, 0, 190]
    off = _offsets(sizes)
    R, H, G, I = off[-1], 256, len(sizes), 256
    dy = torch.randn(R, H, device="cuda").bfloat16()
    wd = (torch.randn(G, H, I, device="cuda") / H**0.5).bfloat16()
    gu = torch.randn(R, 2 * I, device="cuda").bfloat16()
    row_w = torch.rand(R, device="cuda")
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    st = _status()
    dgu, hw, row_dw = gg_swiglu_bwd(dy, wd, go, gu, row_w, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    dh = torch.cat([dy[off[g]:off[g + 1]].float() @ wd[g].float() for g in range(G)])
    g_, u_ = gu[:, :I].float(), gu[:, I:].float()
    s = torch.sigmoid(g_)
    h = g_ * s * u_
    dhw = dh * row_w[:, None]
    dg = dhw * u_ * s * (1 + g_ * (1 - s))
    du = dhw * g_ * s
    assert _rel_err(dgu[:, :I], dg) < 2e-2
    assert _rel_err(dgu[:, I:], du) < 2e-2
    assert _rel_err(hw, h * row_w[:, None]) < 2e-2
    assert _rel_err(row_dw, (dh * h).sum(1)) < 1e-2


@pytest.mark.parametrize("N", [256, 384])
def test_wgrad_ragged_k(N):
    from spec_ep.ops.grouped_gemm import gg_wgrad

    torch.manual_seed(4)
    sizes = [64, 0, 300, 33, 512]
    off = _offsets(sizes, 64)
    R, M, G = off[-1], 256, len(sizes)
    a = torch.zeros(R, M, device="cuda")
    b = torch.zeros(R, N, device="cuda")
    for g, s in enumerate(sizes):
        a[off[g]:off[g] + s] = torch.randn(s, M, device="cuda")
        b[off[g]:off[g] + s] = torch.randn(s, N, device="cuda")
    a, b = a.bfloat16(), b.bfloat16()
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    st = _status()
    out = gg_wgrad(a, b, go, G, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    ref = torch.stack([a[off[g]:off[g + 1]].float().T @ b[off[g]:off[g + 1]].float() for g in range(G)])
    assert _rel_err(out, ref) < 1e-2
    assert out[1].abs().max().item() == 0.0


def test_large_fwd_perf_sanity():
    """A Qwen3-30B-A3B-sized expert GEMM runs and matches a cuBLAS bf16 reference."""
    from spec_ep.ops.grouped_gemm import gg_swiglu_fwd

    torch.manual_seed(5)
    G, H, I, per = 16, 2048, 768, 2048
    off = _offsets([per] * G)
    a = torch.randn(off[-1], H, device="cuda").bfloat16()
    w = (torch.randn(G, 2 * I, H, device="cuda") / H**0.5).bfloat16()
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    h, gu = gg_swiglu_fwd(a, w, go)
    ref = torch.bmm(a.view(G, per, H), w.transpose(1, 2)).float().reshape(-1, 2 * I)
    torch.cuda.synchronize()
    assert _rel_err(gu, ref) < 1e-2


@pytest.mark.parametrize("kind,M,N,G,mult", [("fp32", 256, 384, 4, 1), ("8bit", 256, 384, 4, 1),
                                              ("8bit", 256, 512, 4, 1), ("8bit", 512, 768, 40, 1),
                                              ("8bit", 256, 512, 4, 8)])
def test_wgrad_adamw_fused_matches_unfused(kind, M, N, G, mult):
    """AdamW applied in the wgrad epilogue == wgrad to HBM followed by the standalone update.

    N = 384 takes 128-column tiles, 512 / 768 take 256-column tiles; G = 40 gives every
    CTA several tiles (the 8-bit epilogue's TMA ring wraps many times); mult = 8 makes the
    reduction long enough (>= 512 rows per group on average) for the three-stage operand
    ring with a two-deep epilogue ring.
    """
    from spec_ep.ops.grouped_gemm import gg_wgrad
    from spec_ep.ops.optim import FusedAdamW

    torch.manual_seed(6)
    sizes = [s * mult for s in ([128, 0, 64, 300] * ((G + 3) // 4))[:G]]
    off = _offsets(sizes, 64)
    R = off[-1]
    a = torch.zeros(R, M, device="cuda")
    b = torch.zeros(R, N, device="cuda")
    for g, s in enumerate(sizes):
        a[off[g]:off[g] + s] = torch.randn(s, M, device="cuda")
        b[off[g]:off[g] + s] = torch.randn(s, N, device="cuda")
    a, b = a.bfloat16(), b.bfloat16()
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    w0 = (torch.randn(G, M, N, device="cuda") * 0.02).bfloat16()
    p1 = torch.nn.Parameter(w0.clone())
    p2 = torch.nn.Parameter(w0.clone())
    p1._sepx_state_precision = kind
    p2._sepx_state_precision = kind
    o1 = FusedAdamW([p1], lr=1e-3, weight_decay=0.1)
    o2 = FusedAdamW([p2], lr=1e-3, weight_decay=0.1)
    st = _status()
    for step in range(3):
        o1.fused_wgrad(p1, a, b, go, st)
        o1.step_count += 1
        g = gg_wgrad(a, b, go, G)
        o2.apply_now(p2, g)
        o2.step_count += 1
    torch.cuda.synchronize()
    assert st.item() == 0
    assert torch.equal(p1.detach(), p2.detach())
    for k_ in o1.state[id(p1)]:
        if torch.is_tensor(o1.state[id(p1)][k_]):
            assert torch.equal(o1.state[id(p1)][k_], o2.state[id(p2)][k_]), k_
    # the empty group still got weight decay + moment decay, and parameters moved
    assert not torch.equal(p1.detach(), w0)


@pytest.mark.parametrize("mode", ["fwd", "dgrad", "swiglu_fwd", "swiglu_bwd", "wgrad"])
def test_cta_pair_tiles_match_single_cta_tiles(mode):
    """The 256-column tiles on CTA pairs (tcgen05.mma.cta_group::2) give the single-CTA
    kernel's result on ragged groups, including groups shorter than one 128-row half."""
    from spec_ep.ops import grouped_gemm as gg
    from spec_ep.ops._ext import load

    C = load()
    torch.manual_seed(5)
    sizes = [300, 0, 64, 1000, 130, 17]
    off = _offsets(sizes, 64 if mode == "wgrad" else 1)
    R, G, K, N, I = off[-1], len(sizes), 512, 512, 256
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    a = torch.randn(R, K, device="cuda").bfloat16()

    def run():
        st = _status()
        if mode == "fwd":
            out = gg.gg_fwd(a, (torch.randn(G, N, K, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
                                / K**0.5).bfloat16(), go, status=st)
        elif mode == "dgrad":
            out = gg.gg_dgrad(a, (torch.randn(G, K, N, device="cuda", generator=torch.Generator("cuda").manual_seed(2))
                                  / K**0.5).bfloat16(), go, status=st)
        elif mode == "swiglu_fwd":
            w = (torch.randn(G, 2 * I, K, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
                 / K**0.5).bfloat16()
            out = torch.cat(gg.gg_swiglu_fwd(a, w, go, status=st), 1)
        elif mode == "swiglu_bwd":
            wd = (torch.randn(G, K, I, device="cuda", generator=torch.Generator("cuda").manual_seed(4))
                  / K**0.5).bfloat16()
            gu = torch.randn(R, 2 * I, device="cuda", generator=torch.Generator("cuda").manual_seed(5)).bfloat16()
            row_w = torch.rand(R, device="cuda", generator=torch.Generator("cuda").manual_seed(6))
            dgu, hw, row_dw = gg.gg_swiglu_bwd(a, wd, go, gu, row_w, status=st)
            out = torch.cat([dgu.float(), hw.float(), row_dw[:, None]], 1)
        else:
            b = torch.randn(R, N, device="cuda", generator=torch.Generator("cuda").manual_seed(7)).bfloat16()
            out = gg.gg_wgrad(a, b, go, G, status=st)
        torch.cuda.synchronize()
        assert st.item() == 0
        return out.float()

    prev = C.gemm_set_pairs(True)
    try:
        paired = run()
        C.gemm_set_pairs(False)
        single = run()
    finally:
        C.gemm_set_pairs(prev)
    valid = torch.ones(paired.shape[0], dtype=torch.bool, device="cuda")
    if mode != "wgrad":  # rows of the ragged layout that belong to no group are not written
        valid[:] = False
        for g, s in enumerate(sizes):
            valid[off[g]:off[g] + s] = True
    torch.testing.assert_close(paired[valid], single[valid], rtol=1e-3, atol=1e-3)
