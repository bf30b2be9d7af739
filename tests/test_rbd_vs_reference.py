"""The reference's own RBD (unmodified, installed under baseline/_ref) against this
framework's ``spec_ep.rbd`` on the same gloo ranks and inputs: identical outputs for a
non-identity expert, with and without the concurrent local/inter-node overlap, on 2
simulated nodes x 2 ranks and 4 x 2. CPU only; skipped when the reference is not
installed."""
import importlib.util
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "spec_ep" / "rbd.py"

pytestmark = pytest.mark.skipif(not REF.exists(), reason="reference not installed under baseline/_ref")


def _load_ref():
    spec = importlib.util.spec_from_file_location("reference_rbd_under_test", REF)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _expert(rows, ids):
    e = ids.to(rows.dtype).unsqueeze(-1)
    return torch.tanh(rows * (e + 1) + e)


def _worker(rank, world, gpn, init_file, q):
    from spec_ep.rbd import RBD_combine_dispatch

    ref = _load_ref()
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        local_group, _ = dist.new_subgroups(group_size=gpn)
        g = torch.Generator().manual_seed(7 + rank)
        T, H, E, k = 48 + 8 * rank, 8, 16, 4  # ragged token counts across ranks
        tokens = torch.randn(T, H, generator=g)
        weights = torch.rand(T, k, generator=g)
        route = torch.rand(T, E, generator=g).topk(k, dim=-1).indices
        for concurrent in (False, True):
            want = ref.RBD_combine_dispatch(tokens, weights, _expert, route, E=E, gpus_per_node=gpn,
                                            local_group=local_group, concurrent=concurrent)
            got = RBD_combine_dispatch(tokens, weights, _expert, route, E=E, gpus_per_node=gpn,
                                       local_group=local_group, concurrent=concurrent)
            torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)
        q.put((rank, "ok"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,gpn", [(4, 2), (8, 2)])
def test_outputs_match_the_reference_rbd(tmp_path, world, gpn):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.spawn(_worker, args=(world, gpn, tmp_path / "init", q), nprocs=world, join=True)
    got = sorted(q.get() for _ in range(world))
    assert got == [(r, "ok") for r in range(world)]
