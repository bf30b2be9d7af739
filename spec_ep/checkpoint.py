"""Checkpoint / resume with expert re-sharding, and HF safetensors export.

Layout of a checkpoint directory::

    meta.json            step, world, model config, placement (expert -> rank map)
    dense.pt             replicated weights + their optimizer state (written by rank 0)
    experts_rank{r}.pt   rank r's expert shards + optimizer state, keyed by global expert id

Loading into the same placement restores every tensor bit for bit. Loading into a
different placement (another world size or a planner-chosen layout) gathers every local
expert from the file of its old owner, so expert weights and their optimizer state follow
the experts. 8-bit optimizer blocks are 32 elements and an expert holds a multiple of 32
values, so block-wise state slices per expert exactly.

The expert optimizer state precision is chosen per world size (fp32 where it fits,
block-wise 8-bit otherwise), so a checkpoint may be resumed at another precision:
``meta.json`` records each expert tensor's precision (``expert_state_precision``) and
``load`` converts every expert's state to the resuming optimizer's precision (8-bit codes
decoded to fp32 moments with the restored weight as the master, or fp32 moments encoded
to 8-bit blocks).

The reference keeps only HF checkpoints (scripts/ds_moe.py:28-34, scripts/hf_qwen.py:26-36);
``export_hf`` writes the transformers safetensors layout of ``Qwen3MoeForCausalLM``.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from .ops.optim import convert_state
from .parallel.placement import Placement, contiguous


def _rank_world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _placement_of(model) -> Placement:
    ep = model.ep
    return ep.placement if ep.placement is not None else contiguous(ep.E, ep.world)


def _expert_state_slices(opt, p, G):
    """Optimizer state of expert parameter ``p`` ([G, ...]) as per-expert tensor lists."""
    st = opt.state[id(p)]
    out = {}
    for k, v in st.items():
        if not torch.is_tensor(v):
            out[k] = v
            continue
        out[k] = list(v.reshape(G, -1).unbind(0))
    return out


def save(path, model, trainer=None, step: int = 0):
    """Collective: every rank writes its expert shard; rank 0 writes the replicated part."""
    rank, world = _rank_world()
    os.makedirs(path, exist_ok=True)
    placement = _placement_of(model)
    local = placement.local_experts[model.ep.rank]
    opt = trainer.opt if trainer is not None else None
    shard = {"experts": local, "layers": []}
    precisions = {}
    for li, layer in enumerate(model.layers):
        entry = {}
        for name in ("w_gu", "w_d"):
            p = getattr(layer, name)
            entry[name] = {e: p.detach()[i].cpu() for i, e in enumerate(local)}
            if opt is not None:
                precisions[f"layers.{li}.{name}"] = opt.state[id(p)]["prec"]
                sl = _expert_state_slices(opt, p, len(local))
                entry[name + ".opt"] = {k: ({e: v[i].cpu() for i, e in enumerate(local)} if isinstance(v, list) else v)
                                        for k, v in sl.items()}
        shard["layers"].append(entry)
    torch.save(shard, os.path.join(path, f"experts_rank{rank}.pt"))
    if rank == 0:
        dense = {n: p.detach().cpu() for n, p in model.named_parameters() if not getattr(p, "_sepx_expert", False)}
        dstate = {}
        if opt is not None:
            for n, p in model.named_parameters():
                if getattr(p, "_sepx_expert", False):
                    continue
                dstate[n] = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in opt.state[id(p)].items()}
        torch.save({"params": dense, "opt": dstate, "opt_step": opt.step_count if opt else 0},
                   os.path.join(path, "dense.pt"))
        meta = {"step": step, "world": world, "config": model.cfg.to_dict(), "placement": placement.to_dict(),
                "expert_state_precision": precisions}
        with open(os.path.join(path, "meta.json"), "w") as f:
            json.dump(meta, f)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


@torch.no_grad()
def load(path, model, trainer=None) -> int:
    """Restore into ``model`` (any placement); returns the saved step."""
    with open(os.path.join(path, "meta.json")) as f:
        meta = json.load(f)
    old = Placement.from_dict(meta["placement"])
    new = _placement_of(model)
    me = model.ep.rank
    need = new.local_experts[me]
    owners = sorted({old.owner[e] for e in need})
    shards = {r: torch.load(os.path.join(path, f"experts_rank{r}.pt"), weights_only=False) for r in owners}
    opt = trainer.opt if trainer is not None else None
    for li, layer in enumerate(model.layers):
        for name in ("w_gu", "w_d"):
            p = getattr(layer, name)
            for i, e in enumerate(need):
                p[i].copy_(shards[old.owner[e]]["layers"][li][name][e])
            if opt is not None and (name + ".opt") in shards[old.owner[need[0]]]["layers"][li]:
                st = opt.state[id(p)]
                rows = {k: v.view(len(need), -1) for k, v in st.items() if torch.is_tensor(v)}
                for i, e in enumerate(need):
                    saved = shards[old.owner[e]]["layers"][li][name + ".opt"]
                    src = {k: (v[e].reshape(-1) if isinstance(v, dict) else v) for k, v in saved.items()}
                    src.setdefault("prec", meta.get("expert_state_precision", {}).get(f"layers.{li}.{name}", "fp32"))
                    src = convert_state(src, st["prec"], p[i].detach().cpu())
                    for k, r in rows.items():
                        r[i].copy_(src[k].reshape(-1))
    dense = torch.load(os.path.join(path, "dense.pt"), weights_only=False)
    params = dict(model.named_parameters())
    for n, t in dense["params"].items():
        params[n].copy_(t)
        if opt is not None and n in dense["opt"]:
            for k, v in dense["opt"][n].items():
                if torch.is_tensor(v):
                    opt.state[id(params[n])][k].copy_(v)
    if opt is not None:
        opt.step_count = dense.get("opt_step", 0)
    return int(meta["step"])


def export_hf(path, model):
    """Write a transformers-layout safetensors file (single GPU or gathered experts)."""
    from safetensors.torch import save_file

    from .integrations.hf_qwen import to_hf_state_dict

    sd = {k: v.contiguous().cpu() for k, v in to_hf_state_dict(model).items()}
    os.makedirs(path, exist_ok=True)
    save_file(sd, os.path.join(path, "model.safetensors"))
    return os.path.join(path, "model.safetensors")
