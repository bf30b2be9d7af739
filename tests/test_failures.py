"""Failure detection without faulting a GPU.

* Host side (gloo ranks on CPU): a rank that never joins makes the others fail with a
  timeout error instead of hanging; bad configurations are rejected before any launch.
* GPU side (2 GPUs, NVLS off): a peer that never publishes its dispatch header makes the
  waiting kernel give up after its deadline, record an error code and return; the host
  raises EPError and the CUDA context stays usable.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rendezvous_worker(rank, port, q):
    if rank == 1:
        return  # this rank never joins
    t0 = time.time()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        q.put(("joined", time.time() - t0))
    except Exception as e:  # expected: timeout
        q.put((type(e).__name__, time.time() - t0))


def test_missing_rank_times_out_on_host():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.spawn(_rendezvous_worker, args=(_free_port(), q), nprocs=2, join=True)
    kind, dt = q.get()
    assert kind != "joined" and dt < 60


def test_bad_configurations_rejected():
    from spec_ep.integrations.ds_moe import load_config
    from spec_ep.parallel.placement import contiguous, plan_balanced

    with pytest.raises(ValueError):
        contiguous(10, 4)  # experts do not split over ranks
    with pytest.raises(ValueError):
        plan_balanced(torch.ones(10), 4)
    with pytest.raises(ValueError):
        load_config({"expert_parallel": {"use_grouped_mm": False}})


def test_corrupt_routing_dump_rejected(tmp_path):
    from spec_ep.parallel.placement import loads_from_routing

    with pytest.raises(ValueError):
        loads_from_routing(torch.randint(0, 8, (4, 3)), 8)  # [T, K] instead of [L, T, K]
    with pytest.raises(ValueError):
        loads_from_routing(torch.full((2, 4, 3), 9), 8)  # expert id out of range


def _peer_timeout_worker(rank, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from spec_ep.parallel.ep import EPError, ExpertParallel

        ep = ExpertParallel(8, 2, 256, max_tokens=64, device=dev, timeout_s=1.0)
        x = torch.randn(64, 256, device=dev).bfloat16()
        te = torch.stack([torch.arange(64) % 8, (torch.arange(64) + 4) % 8], 1).int().to(dev)
        tw = torch.full((64, 2), 0.5, device=dev)
        if rank == 0:
            # rank 1 never dispatches: the receive kernel must give up after ~1 s
            t0 = time.time()
            st = ep.dispatch_fwd(x, te, tw)
            torch.cuda.synchronize()
            dt = time.time() - t0
            with pytest.raises(EPError):
                ep.check()
            assert dt < 30
            # the context is still healthy
            y = (x.float() @ x.float().t()).sum()
            assert torch.isfinite(y)
            del st
        dist.barrier()  # between steps, with nothing in flight
        ep.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


@pytest.mark.gpu
def test_peer_never_signals_times_out_on_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_peer_timeout_worker, args=(_free_port(), errq), nprocs=2, join=True)
    assert errq.empty()


@pytest.mark.gpu
def test_corrupted_expert_ids_are_reported_not_followed():
    """A receive-side expert id outside [0, G) is dropped with an error code: no
    out-of-range write happens and ExpertParallel.check() raises."""
    from spec_ep.parallel.ep import EPError, ExpertParallel

    E, k, H, T = 8, 2, 256, 64
    ep = ExpertParallel(E, k, H, max_tokens=T)
    x = torch.randn(T, H, device="cuda").bfloat16()
    te = torch.randint(0, E, (T, k), device="cuda", dtype=torch.int32)
    tw = torch.rand(T, k, device="cuda")
    dst, meta = ep.route_tables(te)
    meta = meta.clone()
    meta[5, 1] = E + 7  # corrupted local expert id
    st = ep.dispatch_fwd(x, te, tw, tables=(dst, meta))
    ep.combine_fwd(st.xp, st)
    torch.cuda.synchronize()
    with pytest.raises(EPError, match="out-of-range local expert"):
        ep.check()
    # the communicator stays usable: a clean layer afterwards reports no error
    st = ep.dispatch_fwd(x, te, tw)
    ep.combine_fwd(st.xp, st)
    ep.check()
    ep.close()


def _placement_worker(rank, port, q):
    from spec_ep.utils.dist import check_placement

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=4,
                            timeout=datetime.timedelta(seconds=30))
    try:
        hosts = check_placement(2)
        errors = []
        for gpn, nodes in ((3, 1), (2, 3)):
            try:
                check_placement(gpn, min_nodes=nodes)
            except RuntimeError as e:
                errors.append(str(e))
        q.put((rank, len(hosts), len(set(hosts)), errors))
    finally:
        dist.destroy_process_group()


def test_check_placement_on_gloo_ranks():
    """4 ranks on one host as 2 nodes x 2: accepted; 3 per node or 3 nodes: rejected."""
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.spawn(_placement_worker, args=(_free_port(), q), nprocs=4, join=True)
    for _ in range(4):
        rank, n, distinct, errors = q.get()
        assert n == 4 and distinct == 1
        assert len(errors) == 2 and "not a multiple" in errors[0] and "at least 3 nodes" in errors[1]
