"""transformers and DeepSpeed-config integrations."""
import json
import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_configs_parse():
    from spec_ep.integrations.ds_moe import load_config

    for name, size in (("qwen_ep4.json", 4), ("qwen_ep8.json", 8)):
        cfg = load_config(os.path.join(ROOT, "configs", name))
        assert cfg.autoep_size == size and cfg.enabled and cfg.preset_model == "qwen3_5_moe"
        assert cfg.micro_batch == 16 and cfg.sepx.dispatch == "p2p"
    cfg = load_config(os.path.join(ROOT, "configs", "qwen3_30b_a3b_ep8_sepx.json"))
    assert cfg.sepx.timeout_us == 10_000_000 and cfg.optimizer["type"] == "AdamW"


def test_config_validation():
    from spec_ep.integrations.ds_moe import load_config

    with pytest.raises(ValueError):
        load_config({"expert_parallel": {"preset_model": "llama"}})
    with pytest.raises(ValueError):
        load_config({"expert_parallel": {"sepx": {"dispatch": "smoke-signals"}}})


def test_hf_config_conversion():
    from spec_ep.integrations.hf_qwen import config_from_hf, random_hf_model

    m = random_hf_model()
    c = config_from_hf(m.config)
    assert (c.num_experts, c.top_k, c.hidden_size, c.head_dim) == (8, 2, 512, 128)


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


def _token_agreement(out, ref, tol=3e-2):
    """Fraction of tokens whose logits match within ``tol`` (relative to the token's max).

    Near-tied router probabilities can pick a different expert for a few tokens when two
    softmax implementations round differently; those tokens then legitimately differ.
    """
    err = (out.float() - ref.float()).abs().amax(-1) / ref.float().abs().amax(-1).clamp_min(1e-6)
    return float((err < tol).float().mean())


@pytest.mark.gpu
def test_swapped_block_matches_hf_experts_with_same_routing():
    """Same routing decisions in, same expert output out (isolates numerics from top-k ties)."""
    from spec_ep.integrations.hf_qwen import SepxQwen3MoeBlock, random_hf_model
    from spec_ep.parallel.ep import ExpertParallel, ep_moe

    m = random_hf_model().cuda().eval()
    block = m.model.layers[0].mlp
    x = torch.randn(256, 512, device="cuda").bfloat16()
    with torch.no_grad():
        _, w, e = block.gate(x)
        ref = block.experts(x, e, w).float()
        ep = ExpertParallel(8, 2, 512, max_tokens=256)
        sb = SepxQwen3MoeBlock.from_hf_block(block, ep)
        out = ep_moe(x, e.int(), w.float(), sb.gate_up_proj, sb.down_proj, ep).float()
    torch.cuda.synchronize()
    ep.check()
    assert _rel(out, ref) < 2e-2
    ep.close()


@pytest.mark.gpu
def test_swapped_hf_blocks_match_hf():
    from spec_ep.integrations.hf_qwen import random_hf_model, swap_moe_blocks
    from spec_ep.parallel.ep import ExpertParallel

    m = random_hf_model().cuda().eval()
    ids = torch.randint(0, 4096, (1, 256), device="cuda")
    with torch.no_grad():
        ref = m(input_ids=ids).logits.float()[0]
        ep = ExpertParallel(8, 2, 512, max_tokens=256)
        assert swap_moe_blocks(m, ep) == 2
        out = m(input_ids=ids).logits.float()[0]
    torch.cuda.synchronize()
    ep.check()
    assert _token_agreement(out, ref) > 0.95
    ep.close()


@pytest.mark.gpu
def test_spec_ep_model_from_hf_matches_hf_logits():
    from spec_ep.integrations.hf_qwen import config_from_hf, from_hf, random_hf_model, to_hf_state_dict
    from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
    from spec_ep.parallel.ep import ExpertParallel

    hf = random_hf_model().cuda().eval()
    cfg = config_from_hf(hf.config)
    ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=256)
    model = Qwen3MoeForCausalLM(cfg, ep)
    from_hf(hf, model)
    ids = torch.randint(0, cfg.vocab_size, (1, 256), device="cuda")
    with torch.no_grad():
        ref = hf(input_ids=ids).logits.float()[0]
        out = model(ids).float()
    torch.cuda.synchronize()
    ep.check()
    assert _token_agreement(out, ref) > 0.95
    sd = to_hf_state_dict(model)
    hsd = hf.state_dict()
    for k, v in sd.items():
        assert torch.equal(v, hsd[k].to(v.dtype)), k
    ep.close()


@pytest.mark.gpu
def test_ds_style_initialize_on_hf_model():
    from spec_ep.integrations.ds_moe import initialize
    from spec_ep.integrations.hf_qwen import random_hf_model

    m = random_hf_model()
    cfg = json.load(open(os.path.join(ROOT, "configs", "qwen3_30b_a3b_ep8_sepx.json")))
    cfg["expert_parallel"]["autoep_size"] = 1
    engine, opt, _, _ = initialize(model=m, config=cfg, max_tokens=128)
    engine.eval()
    with torch.no_grad():
        out = engine(input_ids=torch.randint(0, 4096, (1, 128), device="cuda"), use_cache=False)
    assert out.logits.shape == (1, 128, 4096)
    engine.ep.check()
    engine.ep.close()


def test_sepx_placement_and_engine_options(tmp_path):
    from spec_ep.integrations.ds_moe import _check_engine_options, load_config, plan_placement

    with pytest.raises(ValueError, match="routing_dump"):
        load_config({"expert_parallel": {"sepx": {"replicate_top_k": 4}}})
    with pytest.raises(ValueError):
        load_config({"expert_parallel": {"sepx": {"speculative_slots": -1}}})
    with pytest.raises(ValueError):
        load_config({"expert_parallel": {"sepx": {"speculative_predictor": "oracle"}}})
    assert load_config({"expert_parallel": {"sepx": {"speculative_predictor": "mlp",
                                                     "speculative_interval": 4}}}).sepx.speculative_interval == 4
    for bad in ({"dispatch": "rbd"}, {"groups": 2}):
        with pytest.raises(ValueError):
            _check_engine_options(load_config({"expert_parallel": {"sepx": bad}}))
    # a recorded routing dump ([L, T, K] int16 per rank) drives the placement planner
    g = torch.Generator().manual_seed(0)
    for r in range(2):
        hot = torch.randint(0, 4, (3, 64, 2), generator=g)  # experts 0..3 dominate
        cold = torch.randint(0, 16, (3, 16, 2), generator=g)
        torch.save(torch.cat([hot, cold], 1).to(torch.int16), tmp_path / f"experts_rank{r}.pt")
    cfg = load_config({"expert_parallel": {"sepx": {"routing_dump": str(tmp_path / "experts_rank*.pt"),
                                                    "replicate_top_k": 2}}})
    pl = plan_placement(cfg, 16, 4)
    assert len(pl.replicated) == 2 and set(pl.replicated) <= {0, 1, 2, 3}
    assert sorted(e for r in range(4) for e in pl.local_experts[r] if pl.owner[e] == r) == list(range(16))
    part = plan_placement(load_config({"expert_parallel": {"sepx": {
        "routing_dump": str(tmp_path / "experts_rank*.pt"), "replicate_top_k": 2, "replica_copies": 2}}}), 16, 4)
    assert all(len(part.holders_of(e)) == 2 for e in part.replicated)
    flat = plan_placement(load_config({}), 16, 4)
    assert flat.owner == [e // 4 for e in range(16)]


def test_hf_example_builds_random_or_loaded_weights(tmp_path):
    """examples/hf_qwen.py on the host: random weights from a checkpoint's config by
    default, the checkpoint's own weights with --load-weights (the reference's flag)."""
    import importlib.util

    from spec_ep.integrations.hf_qwen import random_hf_model

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("hf_example", os.path.join(root, "examples", "hf_qwen.py"))
    ex = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ex)
    src = random_hf_model(num_layers=1, hidden=128, experts=4, inter=64, vocab=256, heads=2, kv_heads=1, seed=3)
    src.save_pretrained(tmp_path / "ckpt")
    loaded, tok = ex.build_model(str(tmp_path / "ckpt"), load_weights=True)
    assert tok is None
    w_src = src.model.layers[0].mlp.gate.weight
    assert torch.equal(loaded.model.layers[0].mlp.gate.weight, w_src)
    fresh, _ = ex.build_model(str(tmp_path / "ckpt"), load_weights=False)
    assert fresh.config.num_experts == 4 and fresh.model.layers[0].mlp.gate.weight.shape == w_src.shape
    assert fresh.model.layers[0].self_attn.q_proj.weight.dtype == torch.bfloat16
    assert not torch.equal(fresh.model.layers[0].self_attn.q_proj.weight, src.model.layers[0].self_attn.q_proj.weight)
    with pytest.raises(SystemExit):
        ex.build_model(None, load_weights=True)
