"""CPU / gloo tests of checkpoint re-sharding and optimizer-state precision conversion.

A checkpoint written by two gloo ranks under one placement (contiguous at world 2, or
with replicated hot experts) is loaded into other placements and world sizes on the
host; every expert's weights and optimizer rows must follow the expert. Resuming at
another expert-state precision (8-bit codes <-> fp32 moments) converts the state.
No GPU: the model is a small stand-in with the real parameter layout
(``w_gu [G, 2I, H]``, ``w_d [G, H, I]`` per layer) and the real ``FusedAdamW`` state.
"""
from pathlib import Path
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, H, I, L = 8, 32, 16, 2


class _Model(torch.nn.Module):
    def __init__(self, placement, rank, world):
        super().__init__()
        local = placement.local_experts[rank]
        self.ep = SimpleNamespace(rank=rank, world=world, E=E, placement=placement)
        self.cfg = SimpleNamespace(to_dict=lambda: {"num_experts": E, "hidden_size": H})
        self.layers = torch.nn.ModuleList()
        for li in range(L):
            m = torch.nn.Module()
            m.w_gu = torch.nn.Parameter(torch.stack([_expert_value(li, e, (2 * I, H)) for e in local]))
            m.w_d = torch.nn.Parameter(torch.stack([_expert_value(li, e, (H, I)) for e in local]))
            for p in (m.w_gu, m.w_d):
                p._sepx_expert = True
            m.norm = torch.nn.Parameter(torch.full((H,), 1.0 + li, dtype=torch.bfloat16))
            self.layers.append(m)


def _expert_value(li, e, shape):
    g = torch.Generator().manual_seed(1000 * li + e)
    return (torch.randn(shape, generator=g) + e).bfloat16()


def _trainer(model, prec):
    from spec_ep.ops.optim import FusedAdamW

    experts = [p for p in model.parameters() if getattr(p, "_sepx_expert", False)]
    for p in experts:
        p._sepx_state_precision = prec
    dense = [p for p in model.parameters() if not getattr(p, "_sepx_expert", False)]
    opt = FusedAdamW(dense + experts, state_precision="fp32")
    return SimpleNamespace(opt=opt)


def _fill_state(model, tr, local):
    """Deterministic per-expert optimizer state that identifies the expert."""
    from spec_ep.ops.optim import encode_8bit

    for li, layer in enumerate(model.layers):
        for name in ("w_gu", "w_d"):
            p = getattr(layer, name)
            st = tr.opt.state[id(p)]
            for i, e in enumerate(local):
                m, v = _expert_moments(li, name, e, p[i].numel())
                if st["prec"] == "fp32":
                    st["master"].view(len(local), -1)[i].copy_(p[i].detach().float().reshape(-1))
                    st["m"].view(len(local), -1)[i].copy_(m)
                    st["v"].view(len(local), -1)[i].copy_(v)
                else:
                    mq, ms, vq, vs = encode_8bit(m, v)
                    for k, t in (("mq", mq), ("ms", ms), ("vq", vq), ("vs", vs)):
                        st[k].view(len(local), -1)[i].copy_(t)


def _expert_moments(li, name, e, n):
    g = torch.Generator().manual_seed(7 + 100 * li + 10 * e + (name == "w_d"))
    return torch.randn(n, generator=g) * 1e-3 * (e + 1), torch.rand(n, generator=g) * 1e-6 * (e + 1)


def _save_rank(rank, init_file, path, placement_dict, prec):
    from spec_ep import checkpoint
    from spec_ep.parallel.placement import Placement

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=2)
    placement = Placement.from_dict(placement_dict)
    model = _Model(placement, rank, 2)
    tr = _trainer(model, prec)
    _fill_state(model, tr, placement.local_experts[rank])
    tr.opt.step_count = 5
    checkpoint.save(path, model, tr, step=5)
    dist.destroy_process_group()


def _save(tmp_path, placement, prec):
    tmp_path.mkdir(parents=True, exist_ok=True)
    path = tmp_path / "ck"
    mp.spawn(_save_rank, args=(tmp_path / "init", path, placement.to_dict(), prec), nprocs=2)
    return path


def _check_loaded(path, placement, rank, world, prec, src_prec):
    from spec_ep import checkpoint
    from spec_ep.ops.optim import decode_8bit, encode_8bit

    model = _Model(placement, rank, world)
    with torch.no_grad():
        for p in model.parameters():
            p.zero_()
    tr = _trainer(model, prec)
    assert checkpoint.load(path, model, tr) == 5
    assert tr.opt.step_count == 5
    local = placement.local_experts[rank]
    for li, layer in enumerate(model.layers):
        assert torch.equal(layer.norm, torch.full((H,), 1.0 + li, dtype=torch.bfloat16))
        for name in ("w_gu", "w_d"):
            p = getattr(layer, name)
            st = tr.opt.state[id(p)]
            for i, e in enumerate(local):
                shape = (2 * I, H) if name == "w_gu" else (H, I)
                assert torch.equal(p[i], _expert_value(li, e, shape)), (li, name, e)
                m, v = _expert_moments(li, name, e, p[i].numel())
                if prec == "fp32":
                    if src_prec == "8bit":  # what the checkpoint holds is the 8-bit image of (m, v)
                        m, v = decode_8bit(*encode_8bit(m, v))
                    rows = {k: st[k].view(len(local), -1)[i] for k in ("master", "m", "v")}
                    assert torch.equal(rows["master"], p[i].float().reshape(-1))
                    tol = 0 if src_prec == "fp32" else 1e-6
                    torch.testing.assert_close(rows["m"], m, atol=tol * 1e-3, rtol=tol)
                    torch.testing.assert_close(rows["v"], v, atol=tol * 1e-9, rtol=tol)
                else:
                    mq, ms, vq, vs = encode_8bit(m, v)
                    got = {k: st[k].view(len(local), -1)[i] for k in ("mq", "ms", "vq", "vs")}
                    assert torch.equal(got["mq"], mq) and torch.equal(got["vq"], vq)
                    torch.testing.assert_close(got["ms"], ms)
                    torch.testing.assert_close(got["vs"], vs)


def test_reshard_world2_to_world1_and_world4_same_precision(tmp_path: Path):
    from spec_ep.parallel.placement import contiguous

    path = _save(tmp_path, contiguous(E, 2), "8bit")
    _check_loaded(path, contiguous(E, 1), 0, 1, "8bit", "8bit")
    for r in range(4):
        _check_loaded(path, contiguous(E, 4), r, 4, "8bit", "8bit")


def test_resume_8bit_checkpoint_with_fp32_state_and_back(tmp_path: Path):
    """8-bit state written at world 2 resumes as fp32 state at world 4 (the precision the
    per-world-size choice makes there), and fp32 state resumes as 8-bit."""
    from spec_ep.parallel.placement import contiguous

    path8 = _save(tmp_path / "a", contiguous(E, 2), "8bit")
    for r in range(4):
        _check_loaded(path8, contiguous(E, 4), r, 4, "fp32", "8bit")
    path32 = _save(tmp_path / "b", contiguous(E, 2), "fp32")
    _check_loaded(path32, contiguous(E, 1), 0, 1, "8bit", "fp32")
    import json

    meta = json.loads((path8 / "meta.json").read_text())
    assert set(meta["expert_state_precision"].values()) == {"8bit"}


def test_replicated_placement_reshards_into_contiguous(tmp_path: Path):
    """Shards written under a placement with hot-expert replicas (each rank holds its
    primaries plus copies) load into a plain contiguous placement at world 1 and 4."""
    from spec_ep.parallel.placement import contiguous, plan_balanced

    load = torch.tensor([50.0, 1, 2, 3, 40, 5, 6, 7])
    placement = plan_balanced(load, 2, replicate_top=2)
    assert placement.replicated and all(len(x) > E // 2 for x in placement.local_experts)
    path = _save(tmp_path, placement, "fp32")
    _check_loaded(path, contiguous(E, 1), 0, 1, "fp32", "fp32")
    for r in range(4):
        _check_loaded(path, contiguous(E, 4), r, 4, "fp32", "fp32")


def test_state_codec_roundtrip_bounds():
    """encode_8bit / decode_8bit: m within half a code step, sqrt(v) rounded up (never 0)."""
    from spec_ep.ops.optim import decode_8bit, encode_8bit

    g = torch.Generator().manual_seed(0)
    m = torch.randn(32 * 64, generator=g)
    v = torch.rand(32 * 64, generator=g) ** 4
    v[:32] = 0  # an all-zero block
    mq, ms, vq, vs = encode_8bit(m, v)
    m2, v2 = decode_8bit(mq, ms, vq, vs)
    step_m = (ms / 127).repeat_interleave(32)
    assert (m2 - m).abs().le(step_m * 0.5 + 1e-7).all()
    assert (v2[32:] >= v[32:] * (1 - 1e-6)).all()
    assert torch.equal(v2[:32], torch.zeros(32))
    assert (v2[32:] > 0).all() or (v[32:] == 0).any()
