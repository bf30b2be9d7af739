"""All-to-all NVLink write bandwidth of the two kernel store paths (every rank writes to
every other rank at once, 4 KB rows, destinations interleaved as in the EP dispatch).

  mode 0  SM stores (16-byte vector loads and stores per lane; the EP kernels' path)
  mode 1  TMA bulk copies (cp.async.bulk global -> shared -> peer, 4 rows in flight/warp)

Reports, per mode and grid size, the CUDA-event time (max over ranks) and GB/s sent per
rank (bytes this rank wrote to its peers).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 benchmarks/p2p_store.py [--mib 64]
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--mib", type=int, default=32, help="MiB written to each peer")
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    from spec_ep.parallel.symm import SymmetricBuffer
    from spec_ep.utils.dist import init_distributed

    rank, world, dev = init_distributed()
    per_peer = args.mib << 20
    buf = SymmetricBuffer(per_peer * world, device=dev)
    src = torch.randn(per_peer // 2, device=dev).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    res = []
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for mode in (0, 1):
        for blocks in (sms // 2, sms, 2 * sms):
            def run():
                buf._b.p2p_write_bench(src, per_peer, mode, blocks, status)

            for _ in range(3):
                run()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.iters):
                run()
            e.record()
            e.synchronize()
            t = torch.tensor([s.elapsed_time(e) / args.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
            res.append({"mode": ["sm_store", "tma_bulk"][mode], "blocks": blocks, "ms": ms,
                        "GBps_sent_per_rank": per_peer * (world - 1) / ms / 1e6})
            dist.barrier()
    assert int(status.item()) == 0, "a bulk copy timed out"
    if rank == 0:
        print(json.dumps({"world": world, "MiB_per_peer": args.mib, "results": res}), flush=True)
    buf.barrier()
    buf.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
