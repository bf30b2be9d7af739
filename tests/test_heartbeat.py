"""Host-side liveness (CPU, gloo ranks): a rank that leaves between steps is reported by
name on the other ranks before their next step, within the timeout; no GPU involved."""
import datetime
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from spec_ep.utils.heartbeat import Heartbeat, PeerLostError


def _free_port():
    import socket

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, mode, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    hb = Heartbeat.from_default_group(timeout_s=2.0)
    lost_rank = world - 1
    try:
        for step in range(6):
            hb.arrive(step)
            time.sleep(0.01)  # the step's work
            if rank == lost_rank and step == 2:
                if mode == "crash":
                    q.put((rank, "exited", step))
                    return  # gone after step 2 without a word
                if mode == "drain":
                    hb.leave("drained by the scheduler")
                    q.put((rank, "exited", step))
                    return
        q.put((rank, "done", 6))
    except PeerLostError as e:
        q.put((rank, "lost", e.rank, e.step, e.reason, time.monotonic()))
    # no destroy_process_group: a peer is gone, so the exit barrier would wait for it


def _run(mode, world=3):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    t0 = time.monotonic()
    mp.spawn(_worker, args=(world, _free_port(), mode, q), nprocs=world, join=True)
    out = []
    while not q.empty():
        out.append(q.get())
    return out, time.monotonic() - t0


def test_all_ranks_alive_run_every_step():
    out, _ = _run("healthy")
    assert sorted(o[:2] for o in out) == [(0, "done"), (1, "done"), (2, "done")]


@pytest.mark.parametrize("mode", ["crash", "drain"])
def test_lost_rank_is_named_before_the_next_step(mode):
    out, dt = _run(mode)
    lost = [o for o in out if o[1] == "lost"]
    assert {o[0] for o in lost} == {0, 1}, out
    for _, _, who, step, reason, _ in lost:
        assert who == 2
        # the lost rank does not run step 3: the peers stop before launching it
        assert step == 3
        if mode == "drain":
            assert reason == "left after step 2 (drained by the scheduler)"
        else:
            assert "no heartbeat" in reason and "last arrived at step 2, step 3 needed" in reason
    assert dt < 60


def test_bad_arguments():
    store = dist.HashStore()
    with pytest.raises(ValueError):
        Heartbeat(store, 0, 2, timeout_s=0)
    hb = Heartbeat(store, 0, 1)
    hb.arrive(0)  # no peers: nothing to wait for
    with pytest.raises(ValueError):
        hb.arrive(0)  # once per step
    hb.arrive(1)
    assert hb.arrived == 2


def test_lag_and_leave_on_one_store():
    """Two ranks' views over one in-process store: the wait, the lag allowance, the
    timeout and the leave record."""
    store = dist.HashStore()
    a, b = Heartbeat(store, 0, 2, timeout_s=0.2), Heartbeat(store, 1, 2, timeout_s=0.2)
    a.beat()
    with pytest.raises(PeerLostError, match="no heartbeat"):
        a.wait(0)  # b has not arrived at step 0
    b.arrive(0)
    a.wait(0)
    a.beat()  # a arrives at step 1; b is still in step 0
    Heartbeat(store, 0, 2, max_lag=1).wait(1)  # one step of lag allowed
    b.leave("done")  # b took part in step 0 only
    with pytest.raises(PeerLostError, match=r"left after step 0 \(done\)"):
        a.wait(1)
