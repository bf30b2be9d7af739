"""Expert-weight transfers between GPUs of one NVSwitch box (reference:
benchmark/internode/expert_send_recv.py, expert_all2all.py, expert_send_recv_parallel.py).

One SwiGLU expert = 3 * hidden * intermediate bf16 values (6 MiB at 2048 x 512).
Patterns, each with NCCL and with copy-engine puts into IPC-mapped peer memory:
  pair   rank 0 -> rank 1
  ring   every rank -> rank + 1 (concurrent)
  all2all  every rank sends n experts split evenly over all other ranks
Reports min/avg/max ms over iterations (max over ranks per iteration) and GB/s per rank.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/expert_transfer.py [--experts 1 2 4 8 16 32]
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run(fn, iters, warmup, dev):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    t = torch.tensor(ts, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, nargs="+", default=[1, 2, 4, 8, 16, 32])
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--intermediate", type=int, default=512)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iterations", type=int, default=5)
    args = ap.parse_args()
    from spec_ep.parallel.symm import SymmetricBuffer
    from spec_ep.utils.dist import init_distributed

    rank, world, dev = init_distributed()
    per = 3 * args.hidden * args.intermediate
    nmax = max(args.experts)
    buf = SymmetricBuffer(nmax * per * 2 * 2, device=dev)  # room for a ring/all2all receive
    results = []
    for n in args.experts:
        numel = n * per
        src = torch.randn(numel, device=dev).bfloat16()
        dst = torch.empty_like(src)
        nbytes = numel * 2
        row = {"experts": n, "MiB": nbytes / 2**20}

        def pair_nccl():
            if rank == 0:
                dist.send(src, 1)
            elif rank == 1:
                dist.recv(dst, 0)

        def pair_p2p():
            if rank == 0:
                buf.put(src, 1, 0)

        nxt, prv = (rank + 1) % world, (rank - 1) % world

        def ring_nccl():
            for r in dist.batch_isend_irecv([dist.P2POp(dist.isend, src, nxt), dist.P2POp(dist.irecv, dst, prv)]):
                r.wait()

        def ring_p2p():
            buf.put(src, nxt, 0)

        chunk = numel // max(world - 1, 1)
        splits = [0 if r == rank else chunk for r in range(world)]
        a2a_src = src[: chunk * (world - 1)].contiguous()
        a2a_dst = torch.empty_like(a2a_src)

        def a2a_nccl():
            dist.all_to_all_single(a2a_dst, a2a_src, splits, splits)

        def a2a_p2p():
            j = 0
            for r in range(world):
                if r == rank:
                    continue
                buf.put(a2a_src[j * chunk:(j + 1) * chunk], r, (rank if rank < r else rank - 1) * chunk * 2)
                j += 1

        for name, fn, moved in (("pair_nccl", pair_nccl, nbytes), ("pair_p2p", pair_p2p, nbytes),
                                ("ring_nccl", ring_nccl, nbytes), ("ring_p2p", ring_p2p, nbytes),
                                ("all2all_nccl", a2a_nccl, chunk * (world - 1) * 2),
                                ("all2all_p2p", a2a_p2p, chunk * (world - 1) * 2)):
            if world < 2:
                continue
            ts = run(fn, args.iterations, args.warmup, dev)
            avg = sum(ts) / len(ts)
            row[name] = {"min_ms": min(ts), "avg_ms": avg, "max_ms": max(ts), "GBps_per_rank": moved / avg / 1e6}
        results.append(row)
    if rank == 0:
        print(json.dumps({"world": world, "results": results}, indent=1), flush=True)
    buf.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
