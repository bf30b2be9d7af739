"""DeepSpeed-AutoEP-compatible entry point (config files and ``initialize`` call shape).

The reference wraps an HF Qwen MoE model with ``deepspeed.initialize(model=..., config=...)``
and an AutoEP JSON (scripts/ds_moe.py:50-61, configs/qwen_ep{4,8}.json). This module
reads the same JSON keys::

    {"train_micro_batch_size_per_gpu": 16,
     "expert_parallel": {"enabled": true, "autoep_size": 8, "preset_model": "qwen3_5_moe",
                         "use_grouped_mm": true,
                         "sepx": {"dispatch": "p2p", "groups": 1, "fp8": false,
                                  "replicate_top_k": 0, "routing_dump": null,
                                  "speculative_slots": 0, "speculative_min_count": 1,
                                  "speculative_predictor": "router", "speculative_interval": 1,
                                  "timeout_us": 10000000}},
     "optimizer": {"type": "AdamW", "params": {...}}}

and returns ``(engine, optimizer, None, None)``. ``autoep_size`` < world builds
expert-parallel groups of that size (contiguous ranks) and expert-data-parallel groups
across them; dense weights are data-parallel over every rank.

``sepx`` keys: ``fp8`` sends forward rows as e4m3 with 1x128 scales; ``routing_dump``
(a glob or list of ``experts_rank*.pt`` files) plans a load-balanced placement from
recorded routing, with ``replicate_top_k`` hot experts copied to every rank, or to
``replica_copies`` ranks each; ``speculative_slots``
> 0 turns on speculative replication (an LRU cache of that many predicted-hot experts
per layer and rank; inference only). ``dispatch`` must be ``"p2p"`` for the model engine
(``"rbd"`` names the torch reference, ``spec_ep.rbd.RBD_combine_dispatch``, which is an
API rather than an engine), and ``groups`` > 1 (the two-stage path,
``spec_ep.parallel.hierarchical.HierarchicalEP``) is a forward-only layer of its own.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

KNOWN_PRESETS = ("qwen3_moe", "qwen3_5_moe")


@dataclass
class SepxOptions:
    dispatch: str = "p2p"          # "p2p" (fused NVLink kernels) | "rbd" (torch RBD over NCCL)
    groups: int = 1                # logical GPU groups for the two-stage path
    fp8: bool = False              # e4m3 1x128 dispatch payload (forward only)
    replicate_top_k: int = 0       # hot experts replicated (needs routing_dump)
    replica_copies: int = 0        # ranks holding each replicated expert (0: every rank)
    routing_dump: object = None    # glob / list of experts_rank*.pt files for the placement planner
    speculative_slots: int = 0     # LRU replica cache slots per layer and rank (inference)
    speculative_min_count: int = 1  # fewest predicted rows that make an expert worth fetching
    speculative_predictor: str = "router"  # "router" (router on the residual) | "mlp" (online MLP)
    speculative_interval: int = 1  # re-plan each layer's cache every N calls
    timeout_us: int = 10_000_000   # device-side wait limit


@dataclass
class EPConfig:
    micro_batch: int = 1
    enabled: bool = True
    autoep_size: int = 1
    preset_model: str = "qwen3_moe"
    use_grouped_mm: bool = True
    sepx: SepxOptions = field(default_factory=SepxOptions)
    optimizer: dict = field(default_factory=dict)


def load_config(cfg) -> EPConfig:
    """Parse a DeepSpeed-style config (path or dict) and validate the EP keys."""
    if isinstance(cfg, str):
        with open(cfg) as f:
            cfg = json.load(f)
    ep = cfg.get("expert_parallel", {})
    sx = ep.get("sepx", {})
    out = EPConfig(micro_batch=int(cfg.get("train_micro_batch_size_per_gpu", 1)),
                   enabled=bool(ep.get("enabled", True)), autoep_size=int(ep.get("autoep_size", 1)),
                   preset_model=ep.get("preset_model", "qwen3_moe"), use_grouped_mm=bool(ep.get("use_grouped_mm", True)),
                   sepx=SepxOptions(**{k: sx[k] for k in sx if k in SepxOptions.__dataclass_fields__}),
                   optimizer=cfg.get("optimizer", {}))
    if out.preset_model not in KNOWN_PRESETS:
        raise ValueError(f"unknown preset_model {out.preset_model!r}; expected one of {KNOWN_PRESETS}")
    if out.sepx.dispatch not in ("p2p", "rbd"):
        raise ValueError("expert_parallel.sepx.dispatch must be 'p2p' or 'rbd'")
    if not out.use_grouped_mm:
        raise ValueError("use_grouped_mm=false is not supported: experts always run as grouped GEMMs")
    sx = out.sepx
    if int(sx.groups) < 1 or int(sx.replicate_top_k) < 0 or int(sx.replica_copies) < 0 or int(sx.speculative_slots) < 0 or \
            int(sx.speculative_min_count) < 1 or int(sx.timeout_us) <= 0:
        raise ValueError("expert_parallel.sepx: groups >= 1, replicate_top_k >= 0, speculative_slots >= 0, "
                         "speculative_min_count >= 1 and timeout_us > 0 are required")
    if sx.speculative_predictor not in ("router", "mlp") or int(sx.speculative_interval) < 1:
        raise ValueError("expert_parallel.sepx: speculative_predictor must be 'router' or 'mlp' and "
                         "speculative_interval >= 1")
    if sx.replicate_top_k and not sx.routing_dump:
        raise ValueError("expert_parallel.sepx.replicate_top_k needs measured routing: set sepx.routing_dump")
    return out


def plan_placement(cfg: EPConfig, num_experts: int, world: int):
    """Placement for the EP group: planned from ``sepx.routing_dump`` (expert loads summed
    over layers, ``replicate_top_k`` hot experts on every rank), else contiguous."""
    import glob

    from ..parallel.placement import contiguous, loads_from_routing, plan_balanced
    from ..utils.profile import load_routing

    dump = cfg.sepx.routing_dump
    if not dump:
        return contiguous(num_experts, world)
    files = sorted(glob.glob(dump)) if isinstance(dump, str) else list(dump)
    if not files:
        raise FileNotFoundError(f"sepx.routing_dump matches no files: {dump!r}")
    loads = loads_from_routing(load_routing(files), num_experts).sum(0)
    copies = int(cfg.sepx.replica_copies) or None
    return plan_balanced(loads, world, int(cfg.sepx.replicate_top_k), copies)


def _check_engine_options(cfg: EPConfig):
    if cfg.sepx.dispatch != "p2p":
        raise ValueError("the model engine dispatches with the fused p2p kernels (sepx.dispatch='p2p'); "
                         "spec_ep.rbd.RBD_combine_dispatch is the torch reference API")
    if int(cfg.sepx.groups) > 1:
        raise ValueError("sepx.groups > 1: the two-stage path (spec_ep.parallel.hierarchical.HierarchicalEP) is a "
                         "forward-only layer of its own; the model engine uses the flat path")


def make_groups(autoep_size: int):
    """(ep_group, expert_dp_group): EP over contiguous blocks of ``autoep_size`` ranks,
    expert-data-parallel over ranks holding the same experts. Collective."""
    if not (dist.is_available() and dist.is_initialized()):
        return None, None
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % autoep_size:
        raise ValueError(f"world {world} is not a multiple of autoep_size {autoep_size}")
    ep_group = dp_group = None
    for start in range(0, world, autoep_size):
        g = dist.new_group(list(range(start, start + autoep_size)))
        if start <= rank < start + autoep_size:
            ep_group = g
    n_rep = world // autoep_size
    for off in range(autoep_size):
        ranks = [off + i * autoep_size for i in range(n_rep)]
        g = dist.new_group(ranks)
        if rank in ranks:
            dp_group = g
    return ep_group, (dp_group if n_rep > 1 else None)


class SepxEngine:
    """Minimal engine with the call shape the reference uses (``engine(**batch)``)."""

    def __init__(self, module, trainer=None, ep=None, config: EPConfig | None = None):
        self.module, self.trainer, self.ep, self.config = module, trainer, ep, config
        self.device = ep.device if ep is not None else torch.device("cuda", torch.cuda.current_device())

    def __call__(self, *args, **kwargs):
        if not hasattr(self.module, "generate"):  # spec_ep model: token ids (+ labels) only
            for k in ("use_cache", "attention_mask"):
                kwargs.pop(k, None)
        return self.module(*args, **kwargs)

    def eval(self):
        self.module.eval()
        return self

    def train(self, mode: bool = True):
        self.module.train(mode)
        return self

    def train_step(self, input_ids, labels, num_valid=None):
        if self.trainer is None:
            raise RuntimeError("engine was initialised without an optimizer")
        return self.trainer.train_step(input_ids, labels, num_valid)


def initialize(model=None, config=None, max_tokens: int = 4096, device=None):
    """DeepSpeed-style initialisation.

    ``model``: a transformers Qwen3-MoE / Qwen3.5-MoE model (its MoE blocks are swapped
    for the fused EP layer), a ``spec_ep`` config name, or None to build the preset's
    Qwen3-MoE-shaped ``spec_ep`` model. Returns ``(engine, optimizer, None, None)``.
    """
    from ..parallel.ep import ExpertParallel

    cfg = load_config(config if config is not None else {})
    _check_engine_options(cfg)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    ep_group, dp_group = make_groups(cfg.autoep_size) if cfg.enabled else (None, None)
    world = dist.get_world_size(ep_group) if (dist.is_available() and dist.is_initialized()) else 1
    opt_params = cfg.optimizer.get("params", {})

    if model is None or isinstance(model, str):
        from ..models.config import get_config
        from ..models.qwen3_moe import Qwen3MoeForCausalLM
        from ..train import Trainer

        mcfg = get_config(model or "qwen3-30b-a3b")
        placement = plan_placement(cfg, mcfg.num_experts, world)
        ep = ExpertParallel(mcfg.num_experts, mcfg.top_k, mcfg.hidden_size, max_tokens, group=ep_group,
                            placement=placement, timeout_s=cfg.sepx.timeout_us * 1e-6, device=device,
                            fp8_dispatch=bool(cfg.sepx.fp8))
        net = Qwen3MoeForCausalLM(mcfg, ep, device=device)
        if cfg.sepx.speculative_slots:  # inference engine: no optimizer
            from ..parallel.speculative import enable_speculation

            enable_speculation(net, int(cfg.sepx.speculative_slots), int(cfg.sepx.speculative_min_count),
                               predictor=cfg.sepx.speculative_predictor,
                               interval=int(cfg.sepx.speculative_interval))
            return SepxEngine(net, None, ep, cfg), None, None, None
        tr = Trainer(net, lr=opt_params.get("lr", 1e-4), betas=tuple(opt_params.get("betas", (0.9, 0.95))),
                     weight_decay=opt_params.get("weight_decay", 0.1), expert_dp_group=dp_group)
        return SepxEngine(net, tr, ep, cfg), tr.opt, None, None

    from .hf_qwen import swap_moe_blocks

    c = getattr(model.config, "text_config", model.config)
    if cfg.sepx.speculative_slots:
        raise ValueError("sepx.speculative_slots applies to spec_ep models (Qwen3MoeForCausalLM), not HF blocks")
    ep = ExpertParallel(c.num_experts, c.num_experts_per_tok, c.hidden_size, max_tokens, group=ep_group,
                        placement=plan_placement(cfg, c.num_experts, world), timeout_s=cfg.sepx.timeout_us * 1e-6,
                        device=device, fp8_dispatch=bool(cfg.sepx.fp8))
    model.to(device=device, dtype=torch.bfloat16)
    n = swap_moe_blocks(model, ep)
    if n == 0:
        raise ValueError("no Qwen3-MoE sparse blocks found to swap")
    return SepxEngine(model, None, ep, cfg), None, None, None
