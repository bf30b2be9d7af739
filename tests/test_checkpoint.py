"""Checkpoint / resume and HF export (one GPU)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _tiny(ep_kwargs=None):
    from spec_ep.models.config import get_config
    from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
    from spec_ep.parallel.ep import ExpertParallel
    from spec_ep.train import Trainer

    cfg = get_config("tiny")
    ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=128, **(ep_kwargs or {}))
    torch.manual_seed(0)
    model = Qwen3MoeForCausalLM(cfg, ep)
    tr = Trainer(model, lr=1e-3, expert_state="8bit")
    return cfg, ep, model, tr


def _step(cfg, tr):
    ids = torch.randint(0, cfg.vocab_size, (1, 128), device="cuda")
    lab = torch.cat([ids[:, 1:], torch.full((1, 1), -1, device="cuda")], 1).int()
    return float(tr.train_step(ids, lab, 127))


def test_save_load_roundtrip_is_exact(tmp_path):
    from spec_ep import checkpoint

    cfg, ep, model, tr = _tiny()
    _step(cfg, tr)
    checkpoint.save(tmp_path / "ck", model, tr, step=1)
    ref = {n: p.detach().clone() for n, p in model.named_parameters()}
    ref_state = {id_: {k: v.clone() for k, v in st.items() if torch.is_tensor(v)} for id_, st in tr.opt.state.items()}
    _step(cfg, tr)  # move away from the checkpoint
    assert any(not torch.equal(p, ref[n]) for n, p in model.named_parameters())
    assert checkpoint.load(tmp_path / "ck", model, tr) == 1
    for n, p in model.named_parameters():
        assert torch.equal(p, ref[n]), n
    for id_, st in tr.opt.state.items():
        for k, v in ref_state[id_].items():
            assert torch.equal(st[k], v), k
    ep.close()


def test_export_hf_safetensors(tmp_path):
    from safetensors.torch import load_file

    from spec_ep import checkpoint
    from spec_ep.integrations.hf_qwen import to_hf_state_dict

    cfg, ep, model, tr = _tiny()
    f = checkpoint.export_hf(tmp_path / "hf", model)
    sd = load_file(f)
    ref = to_hf_state_dict(model)
    assert set(sd) == set(ref)
    for k in ref:
        assert torch.equal(sd[k], ref[k].cpu()), k
    assert sd["model.layers.0.mlp.experts.gate_up_proj"].shape == (cfg.num_experts, 2 * cfg.moe_intermediate_size,
                                                                   cfg.hidden_size)
    ep.close()
