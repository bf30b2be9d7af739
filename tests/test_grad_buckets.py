"""Overlapped dense-gradient averaging (spec_ep.train._GradBuckets) on 2 gloo ranks (CPU)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spec_ep.train import _GradBuckets

        torch.manual_seed(0)  # identical parameters on every rank
        params = [torch.nn.Parameter(torch.randn(n)) for n in (5, 17, 64, 3, 40)]
        unused = params[3]
        # small buckets so several all-reduces run during the backward pass
        buckets = _GradBuckets(params, None, bucket_bytes=128)
        assert len(buckets.buckets) > 1
        for step in range(2):
            g = torch.Generator().manual_seed(100 * step + rank)
            xs = [torch.randn(p.numel(), generator=g) for p in params]
            buckets.begin()
            loss = sum((p * x).sum() for p, x in zip(params, xs) if p is not unused)
            loss.backward()
            buckets.finish()
            got = [p.grad.clone() for p in params]
            for p in params:
                p.grad = None
            # expected: mean over ranks of x (d loss / d p = x), zero for the unused one
            allx = [torch.zeros(world, p.numel()) for p in params]
            for r in range(world):
                gr = torch.Generator().manual_seed(100 * step + r)
                for k, p in enumerate(params):
                    allx[k][r] = torch.randn(p.numel(), generator=gr)
            for k, p in enumerate(params):
                want = torch.zeros(p.numel()) if p is unused else allx[k].mean(0)
                torch.testing.assert_close(got[k], want)
        # a backward pass outside begin/finish leaves .grad alone
        (params[0] * 2).sum().backward()
        assert torch.equal(params[0].grad, torch.full((5,), 2.0))
        out[rank] = True
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def test_grad_buckets_average_two_ranks():
    world, port = 2, _free_port()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    assert all(out.get(r) for r in range(world))
