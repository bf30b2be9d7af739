"""Rank / environment helpers (reference: src/utils.py:6-27, benchmark/utils.py:9-51).

Accepts both torchrun (``RANK``/``WORLD_SIZE``/``LOCAL_RANK``) and SLURM
(``SLURM_PROCID``/``SLURM_NTASKS``/``SLURM_LOCALID``) environments.
"""
from __future__ import annotations

import datetime
import os
import socket

import torch
import torch.distributed as dist


def get_rank_and_world_size() -> tuple[int, int]:
    """Export torchrun-style variables from SLURM's when missing; return (rank, world)."""
    if "RANK" not in os.environ and "SLURM_PROCID" in os.environ:
        os.environ["RANK"] = os.environ["SLURM_PROCID"]
        os.environ["WORLD_SIZE"] = os.environ["SLURM_NTASKS"]
        os.environ["LOCAL_RANK"] = os.environ.get("SLURM_LOCALID", "0")
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def local_rank() -> int:
    get_rank_and_world_size()
    return int(os.environ.get("LOCAL_RANK", "0"))


def print0(*msg, **kw):
    """Print on global rank 0 only."""
    rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else get_rank_and_world_size()[0]
    if rank == 0:
        print(*msg, flush=True, **kw)


def init_distributed(backend: str | None = None, timeout_s: float = 600.0):
    """Initialise the default process group from the environment; returns (rank, world, device).

    NCCL on GPUs (one process per GPU, ``device_id`` bound) and gloo otherwise. A short
    ``timeout_s`` makes ranks that wait for a lost peer fail with an error.
    """
    rank, world = get_rank_and_world_size()
    if torch.cuda.is_available():
        lr = local_rank()
        torch.cuda.set_device(lr)
        dev = torch.device("cuda", lr)
    else:
        dev = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        backend = backend or ("nccl" if dev.type == "cuda" else "gloo")
        kw = dict(timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = dev
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        dist.init_process_group(backend, **kw)
    return rank, world, dev


def shutdown_comm():
    """Barrier then destroy, so ranks do not race on rank 0's store at exit (src/utils.py:10-14)."""
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def check_placement(gpus_per_node: int, min_nodes: int = 1) -> list[str]:
    """Check ranks fill nodes in contiguous blocks of ``gpus_per_node``; return every rank's host.

    Mirrors benchmark/utils.py:27-51; ``min_nodes=2`` reproduces its multi-node requirement.
    """
    world = dist.get_world_size()
    if world % gpus_per_node:
        raise RuntimeError(f"{world} ranks is not a multiple of {gpus_per_node} per node.")
    nodes = world // gpus_per_node
    if nodes < min_nodes:
        raise RuntimeError(f"Expected at least {min_nodes} nodes, got {nodes}.")
    hosts = [None] * world
    dist.all_gather_object(hosts, socket.gethostname())
    for n in range(nodes):
        block = hosts[n * gpus_per_node:(n + 1) * gpus_per_node]
        if len(set(block)) != 1:
            raise RuntimeError(f"ranks of node {n} are on different hosts: {block}")
    return hosts
