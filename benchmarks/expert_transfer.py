"""Expert-weight transfers between GPUs of one NVSwitch box (reference:
benchmark/internode/expert_send_recv.py, expert_all2all.py, expert_send_recv_parallel.py).

One SwiGLU expert = 3 * hidden * intermediate values (6 MiB in bf16 at 2048 x 512). The
box's GPUs are split into logical groups of ``--group-size`` ranks, which stand for the
reference's nodes: the "remote" patterns move bytes between groups only.

  pair      rank 0 -> rank 1 (NCCL send/recv | copy-engine put into peer memory)
  ring      every rank -> the same local rank of the next group, concurrently
            (NCCL batch_isend_irecv | copy-engine put)
  all2all   every rank sends n experts split over every rank of the other groups; with
            --balance uneven_internode the first half of the groups send n * (1 + delta)
            experts and the rest n * (1 - delta), with uneven_intranode the first half of
            the local ranks of every group (NCCL all_to_all_single | copy-engine puts)
  sm_pull   every rank pulls n experts from the same local rank of the next group with
            the kernel that fills the speculative replica cache (16-byte peer loads)

Reports min / avg / max ms over iterations (each the max over ranks, CUDA events) and
GB/s per rank of the bytes each rank sends.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/expert_transfer.py \\
        [--experts 1 2 4 8 16 32] [--group-size 4] [--balance even|uneven_internode|uneven_intranode]
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


def group_splits(numel, rank, world, group_size, balance, delta):
    """(send, recv) element counts per rank for the cross-group all-to-all.

    Ranks of the own group get nothing. Every rank's payload is ``numel`` (even) or
    ``numel * (1 +/- delta)`` (heavy / light ranks), split equally over the ranks of the
    other groups; a receiver gets each sender's per-rank share.
    """
    groups = world // group_size
    remote = world - group_size
    if remote == 0:
        raise ValueError("all2all needs at least two groups")
    mine = rank // group_size

    def heavy(r):
        if balance == "uneven_internode":
            if groups % 2:
                raise ValueError(f"uneven_internode needs an even number of groups, got {groups}")
            return r // group_size < groups // 2
        if balance == "uneven_intranode":
            if group_size % 2:
                raise ValueError(f"uneven_intranode needs an even group size, got {group_size}")
            return r % group_size < group_size // 2
        return None

    def share(r):
        h = heavy(r)
        total = numel if h is None else numel * (1 + delta if h else 1 - delta)
        per = total / remote
        if per != int(per):
            raise ValueError(f"{total} elements do not split over {remote} ranks")
        return int(per)

    send = [0 if r // group_size == mine else share(rank) for r in range(world)]
    recv = [0 if r // group_size == mine else share(r) for r in range(world)]
    return send, recv


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--experts", type=int, nargs="+", default=[1, 2, 4, 8, 16, 32])
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--intermediate", type=int, default=512)
    ap.add_argument("--dtype", choices=["bfloat16", "float16", "float32"], default="bfloat16")
    ap.add_argument("--group-size", type=int, default=0, help="ranks per logical group (default: world / 2)")
    ap.add_argument("--balance", choices=["even", "uneven_internode", "uneven_intranode"], default="even")
    ap.add_argument("--load-delta", type=float, default=0.5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iterations", type=int, default=5)
    args = ap.parse_args()
    from spec_ep.parallel.symm import SymmetricBuffer
    from spec_ep.utils.dist import init_distributed

    rank, world, dev = init_distributed()
    if world < 2:
        raise SystemExit("expert_transfer needs at least 2 ranks")
    gs = args.group_size or max(world // 2, 1)
    if world % gs:
        raise SystemExit(f"world {world} is not a multiple of --group-size {gs}")
    dtype = getattr(torch, args.dtype)
    esize = torch.tensor([], dtype=dtype).element_size()
    per = 3 * args.hidden * args.intermediate
    nmax = max(args.experts)
    remote = world - gs
    # receive room: [0, big) for pair / ring puts and the pull's 2 * n expert slots, then
    # one share per sender for the all-to-all puts
    big = 2 * nmax * per
    share_max = int(nmax * per * (1 + args.load_delta)) // max(remote, 1) + 1
    buf = SymmetricBuffer((big + world * share_max) * esize, device=dev)
    results = []
    nxt = (rank + gs) % world  # same local rank, next group
    prv = (rank - gs) % world
    for n in args.experts:
        numel = n * per
        src = torch.randn(numel, device=dev).to(dtype)
        dst = torch.empty_like(src)
        nbytes = numel * esize
        row = {"experts": n, "MiB": nbytes / 2**20, "group_size": gs, "balance": args.balance}

        def pair_nccl():
            if rank == 0:
                dist.send(src, 1)
            elif rank == 1:
                dist.recv(dst, 0)

        def pair_p2p():
            if rank == 0:
                buf.put(src, 1, 0)

        def ring_nccl():
            for r in dist.batch_isend_irecv([dist.P2POp(dist.isend, src, nxt), dist.P2POp(dist.irecv, dst, prv)]):
                r.wait()

        def ring_p2p():
            buf.put(src, nxt, 0)

        patterns = [("pair_nccl", pair_nccl, nbytes), ("pair_p2p", pair_p2p, nbytes)]
        if world // gs >= 2:
            patterns += [("ring_nccl", ring_nccl, nbytes), ("ring_p2p", ring_p2p, nbytes)]
            send, recv = group_splits(numel, rank, world, gs, args.balance, args.load_delta)
            a2a_src = torch.randn(sum(send), device=dev).to(dtype)
            a2a_dst = torch.empty(sum(recv), device=dev, dtype=dtype)
            slot = max(max(send), max(recv))

            def a2a_nccl():
                dist.all_to_all_single(a2a_dst, a2a_src, recv, send)

            def a2a_p2p():
                off = 0
                for r in range(world):
                    if send[r]:
                        buf.put(a2a_src[off:off + send[r]], r, (big + rank * slot) * esize)
                        off += send[r]

            patterns += [("all2all_nccl", a2a_nccl, sum(send) * esize), ("all2all_p2p", a2a_p2p, sum(send) * esize)]
            if (per * esize) % 16 == 0:
                # n pinned experts in slots [0, n), pulled into slots [n, 2n) of the puller
                fr = torch.full((n,), nxt, dtype=torch.int32, device=dev)
                fs = torch.arange(n, dtype=torch.int32, device=dev)

                def sm_pull():
                    buf._b.fetch_experts(n, n, [0], [per * esize], fr, fs, max(1, 128 // n))

                patterns.append(("sm_pull", sm_pull, nbytes))
        for name, fn, moved in patterns:
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
