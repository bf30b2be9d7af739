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


def test_same_api_surface_as_the_reference():
    """Every function and plan type of the reference's rbd module exists here with the
    same parameters in the same order (NamedTuple fields included), and the two plan
    helpers agree on random inputs."""
    import inspect

    import spec_ep.rbd as ours

    ref = _load_ref()
    for name, obj in vars(ref).items():
        if name.startswith("__") or getattr(obj, "__module__", "") != ref.__name__:
            continue
        if not (inspect.isfunction(obj) or inspect.isclass(obj)):
            continue
        mine = getattr(ours, name)
        if hasattr(obj, "_fields"):
            assert mine._fields == obj._fields, name
        if inspect.isfunction(obj):
            want = [p.name for p in inspect.signature(obj).parameters.values()]
            got = [p.name for p in inspect.signature(mine).parameters.values()][:len(want)]
            assert got == want, name
    g = torch.Generator().manual_seed(3)
    counts = torch.randint(0, 9, (6,), generator=g)
    assert torch.equal(ours._start_offsets(counts), ref._start_offsets(counts))
    rows, w, e = torch.arange(40), torch.rand(40, generator=g), torch.randint(0, 16, (40,), generator=g)
    for a, b in zip(ours._sort_copies(rows, w, e, 4, 2), ref._sort_copies(rows, w, e, 4, 2)):
        assert torch.equal(a, b)
