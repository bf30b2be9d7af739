"""Expert parallelism over NVLink peer memory on 2+ GPUs (child processes, NCCL bootstrap).

Each rank holds E / world experts; outputs and gradients are compared with an fp32
single-process reference that holds all experts.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


def _moe_ref(x, te, tw, w_gu, w_d):
    I = w_d.shape[2]
    out = torch.zeros(x.shape, device=x.device)
    for j in range(te.shape[1]):
        for e in te[:, j].unique().tolist():
            m = te[:, j] == e
            gu = x[m] @ w_gu[e].t()
            out[m] += tw[m, j:j + 1] * ((torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]) @ w_d[e].t())
    return out


def _worker(rank, world, port, T, E, k, H, I, skew, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.parallel.ep import ExpertParallel, ep_moe

        g = torch.Generator().manual_seed(0)
        w_gu_full = (torch.randn(E, 2 * I, H, generator=g) / H**0.5).bfloat16().to(dev)
        w_d_full = (torch.randn(E, H, I, generator=g) / I**0.5).bfloat16().to(dev)
        epr = E // world
        w_gu = w_gu_full[rank * epr:(rank + 1) * epr].clone().requires_grad_()
        w_d = w_d_full[rank * epr:(rank + 1) * epr].clone().requires_grad_()
        torch.manual_seed(10 + rank)
        x = torch.randn(T, H, device=dev).bfloat16().requires_grad_()
        logits = torch.randn(T, E, device=dev)
        if skew:  # make rank 0's experts hot
            logits[:, :epr] += 2.0
        p = torch.softmax(logits, -1)
        tw, te = p.topk(k, -1)
        tw = (tw / tw.sum(-1, keepdim=True)).requires_grad_()
        ep = ExpertParallel(E, k, H, max_tokens=T, device=dev, capacity_factor=float(world))
        for _ in range(2):  # run twice: epochs advance, buffers are reused
            out = ep_moe(x, te.int(), tw, w_gu, w_d, ep)
            gout = torch.randn(out.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(rank))
            x.grad = tw.grad = w_gu.grad = w_d.grad = None
            out.backward(gout.bfloat16())
        torch.cuda.synchronize()
        ep.check()
        xr = x.detach().float().requires_grad_()
        twr = tw.detach().clone().requires_grad_()
        gur = w_gu_full.float().requires_grad_()
        dr = w_d_full.float().requires_grad_()
        ref = _moe_ref(xr, te, twr, gur, dr)
        ref.backward(gout.bfloat16().float())
        gg, dd = gur.grad.clone(), dr.grad.clone()
        dist.all_reduce(gg)
        dist.all_reduce(dd)
        assert _rel(out, ref) < 2e-2, _rel(out, ref)
        assert _rel(x.grad, xr.grad) < 3e-2
        assert _rel(tw.grad, twr.grad) < 3e-2
        assert _rel(w_gu.grad, gg[rank * epr:(rank + 1) * epr]) < 3e-2
        assert _rel(w_d.grad, dd[rank * epr:(rank + 1) * epr]) < 3e-2
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, never hang it
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


@pytest.mark.parametrize("skew,k", [(False, 4), (True, 4), (False, 8)])
def test_ep_moe_two_or_more_gpus(skew, k):
    """k = 8 also covers the packed (vector-store) metadata of the dispatch."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_worker, args=(world, _free_port(), 1024, 16, k, 512, 256, skew, errq), nprocs=world, join=True)
    assert errq.empty()


def _placement_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.parallel.ep import ExpertParallel, ep_moe
        from spec_ep.parallel.placement import plan_balanced

        T, E, k, H, I = 1024, 16, 4, 512, 256
        load = torch.arange(E, 0, -1).double() ** 1.5  # skewed popularity
        plan = plan_balanced(load, world, replicate_top=2)
        g = torch.Generator().manual_seed(0)
        w_gu_full = (torch.randn(E, 2 * I, H, generator=g) / H**0.5).bfloat16().to(dev)
        w_d_full = (torch.randn(E, H, I, generator=g) / I**0.5).bfloat16().to(dev)
        mine = plan.local_experts[rank]
        w_gu = w_gu_full[mine].clone().requires_grad_()
        w_d = w_d_full[mine].clone().requires_grad_()
        torch.manual_seed(20 + rank)
        x = torch.randn(T, H, device=dev).bfloat16().requires_grad_()
        p = torch.softmax(torch.randn(T, E, device=dev) + torch.log(load.float().to(dev)), -1)
        tw, te = p.topk(k, -1)
        tw = (tw / tw.sum(-1, keepdim=True)).requires_grad_()
        ep = ExpertParallel(E, k, H, max_tokens=T, device=dev, placement=plan, capacity_factor=float(world))
        out = ep_moe(x, te.int(), tw, w_gu, w_d, ep)
        gout = torch.randn(out.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(rank))
        out.backward(gout.bfloat16())
        torch.cuda.synchronize()
        ep.check()
        xr = x.detach().float().requires_grad_()
        twr = tw.detach().clone().requires_grad_()
        gur = w_gu_full.float().requires_grad_()
        dr = w_d_full.float().requires_grad_()
        ref = _moe_ref(xr, te, twr, gur, dr)
        ref.backward(gout.bfloat16().float())
        assert _rel(out, ref) < 2e-2
        assert _rel(x.grad, xr.grad) < 3e-2
        assert _rel(tw.grad, twr.grad) < 3e-2
        # expert gradients: sum the local copies' gradients over holders, per global expert
        acc_gu = torch.zeros_like(gur.grad)
        acc_d = torch.zeros_like(dr.grad)
        acc_gu[mine] += w_gu.grad.float()
        acc_d[mine] += w_d.grad.float()
        for t in (acc_gu, acc_d, gur.grad, dr.grad):
            dist.all_reduce(t)
        assert _rel(acc_gu, gur.grad) < 3e-2
        assert _rel(acc_d, dr.grad) < 3e-2
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


def test_ep_moe_balanced_placement_with_replicas():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_placement_worker, args=(world, _free_port(), errq), nprocs=world, join=True)
    assert errq.empty()


def _fp8_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.parallel.ep import ExpertParallel, ep_moe

        T, E, k, H, I = 1024, 16, 4, 1024, 256
        g = torch.Generator().manual_seed(0)
        epr = E // world
        w_gu = (torch.randn(E, 2 * I, H, generator=g) / H**0.5).bfloat16().to(dev)[rank * epr:(rank + 1) * epr]
        w_d = (torch.randn(E, H, I, generator=g) / I**0.5).bfloat16().to(dev)[rank * epr:(rank + 1) * epr]
        torch.manual_seed(30 + rank)
        x = torch.randn(T, H, device=dev).bfloat16()
        tw, te = torch.softmax(torch.randn(T, E, device=dev), -1).topk(k, -1)
        ep16 = ExpertParallel(E, k, H, max_tokens=T, device=dev)
        ep8 = ExpertParallel(E, k, H, max_tokens=T, device=dev, fp8_dispatch=True)
        with torch.no_grad():
            ref = ep_moe(x, te.int(), tw, w_gu.contiguous(), w_d.contiguous(), ep16)
            out = ep_moe(x, te.int(), tw, w_gu.contiguous(), w_d.contiguous(), ep8)
        torch.cuda.synchronize()
        ep16.check()
        ep8.check()
        err = _rel(out, ref)
        assert 0 < err < 0.08, err  # e4m3 payload: small but non-zero error
        dist.barrier()
        ep16.close()
        ep8.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


def test_ep_moe_fp8_dispatch():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_fp8_worker, args=(min(n, 4), _free_port(), errq), nprocs=min(n, 4), join=True)
    assert errq.empty()


def _hier_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.parallel.ep import ExpertParallel, ep_moe
        from spec_ep.parallel.hierarchical import HierarchicalEP

        T, E, k, H, I = 512, 16, 4, 512, 256
        gs = 1 if world == 2 else 2
        torch.manual_seed(40 + rank)
        x = torch.randn(T, H, device=dev).bfloat16()
        tw, te = torch.softmax(torch.randn(T, E, device=dev), -1).topk(k, -1)
        te = te.int()
        hep = HierarchicalEP(E, k, H, max_tokens=T, group_size=gs, device=dev)
        # identity experts: every token comes back as x * sum(weights) (the reference's oracle)
        for _ in range(2):
            out = hep.forward(x, te, tw)
        torch.cuda.synchronize()
        hep.check()
        expect = (x.float() * tw.sum(-1, keepdim=True))
        assert _rel(out, expect) < 2e-2, _rel(out, expect)
        assert int(hep.last_pilot_rows.sum()) > 0  # pilots actually crossed groups
        # real experts: agrees with the flat fused path
        g = torch.Generator().manual_seed(0)
        epr = E // world
        w_gu = (torch.randn(E, 2 * I, H, generator=g) / H**0.5).bfloat16().to(dev)[rank * epr:(rank + 1) * epr].contiguous()
        w_d = (torch.randn(E, H, I, generator=g) / I**0.5).bfloat16().to(dev)[rank * epr:(rank + 1) * epr].contiguous()
        flat = ExpertParallel(E, k, H, max_tokens=T, device=dev)
        with torch.no_grad():
            ref = ep_moe(x, te, tw, w_gu, w_d, flat)
        out2 = hep.forward(x, te, tw, w_gu, w_d)
        torch.cuda.synchronize()
        hep.check()
        flat.check()
        assert _rel(out2, ref) < 3e-2, _rel(out2, ref)
        dist.barrier()
        hep.close()
        flat.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


def test_hierarchical_two_stage_dispatch():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 4 if n >= 4 else 2
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_hier_worker, args=(world, _free_port(), errq), nprocs=world, join=True)
    assert errq.empty()


def _graph_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.ops.grouped_gemm import gg_fwd, gg_swiglu_fwd
        from spec_ep.parallel.ep import EPGraph, ExpertParallel

        T, E, k, H, I = 128, 16, 4, 512, 256
        g = torch.Generator().manual_seed(0)
        epr = E // world
        w_gu = (torch.randn(E, 2 * I, H, generator=g) / H**0.5).bfloat16()[rank * epr:(rank + 1) * epr].to(dev)
        w_d = (torch.randn(E, H, I, generator=g) / I**0.5).bfloat16()[rank * epr:(rank + 1) * epr].to(dev)

        def layers(ep, x, te, tw, static):
            for _ in range(2):
                st = ep.dispatch_fwd(x, te, tw, static_rows=static)
                h, _ = gg_swiglu_fwd(st.xp, w_gu, st.group_off, status=ep.status)
                x = ep.combine_fwd(gg_fwd(h, w_d, st.group_off, status=ep.status), st)
            return x

        def inputs(seed):
            gg = torch.Generator(device=dev).manual_seed(1000 * seed + rank)
            x = torch.randn(T, H, device=dev, generator=gg).bfloat16()
            tw, te = torch.softmax(torch.randn(T, E, device=dev, generator=gg), -1).topk(k, -1)
            return x, te.int(), tw

        eager_ep = ExpertParallel(E, k, H, max_tokens=T, device=dev)
        graph_ep = ExpertParallel(E, k, H, max_tokens=T, device=dev)
        xs, tes, tws = inputs(0)
        graph = EPGraph(graph_ep, lambda: layers(graph_ep, xs, tes, tws, True))
        for seed in (1, 2, 3):  # every replay runs under a new device-side epoch
            x, te, tw = inputs(seed)
            xs.copy_(x)
            tes.copy_(te)
            tws.copy_(tw)
            got = graph.replay().clone()
            want = layers(eager_ep, x, te, tw, False)
            torch.cuda.synchronize()
            assert torch.equal(got, want), seed
        graph_ep.check()
        eager_ep.check()
        dist.barrier()
        del graph
        graph_ep.close()
        eager_ep.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


def test_ep_layers_cuda_graph_across_gpus():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_graph_worker, args=(world, _free_port(), errq), nprocs=world, join=True)
    assert errq.empty()


def _replica_train_worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.models.config import get_config
        from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
        from spec_ep.parallel.ep import ExpertParallel
        from spec_ep.parallel.placement import plan_balanced
        from spec_ep.train import Trainer

        cfg = get_config("tiny", num_experts=8, top_k=2)
        T = 256
        load = torch.tensor([40., 30, 5, 4, 3, 2, 1, 1])
        pl = plan_balanced(load, world, replicate_top=2)
        ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=T, device=dev, placement=pl)
        torch.manual_seed(0)
        model = Qwen3MoeForCausalLM(cfg, ep, device=dev)
        g = torch.Generator().manual_seed(1)
        I, H = cfg.moe_intermediate_size, cfg.hidden_size
        full_gu = (torch.randn(cfg.num_experts, 2 * I, H, generator=g) * 0.02).bfloat16()
        full_d = (torch.randn(cfg.num_experts, H, I, generator=g) * 0.02).bfloat16()
        mine = pl.local_experts[rank]
        with torch.no_grad():
            for layer in model.layers:
                layer.w_gu.copy_(full_gu[mine].to(dev))
                layer.w_d.copy_(full_d[mine].to(dev))
                layer.router_logit_bias = torch.linspace(1.0, -1.0, cfg.num_experts, device=dev)
        trainer = Trainer(model, lr=1e-2, expert_state="fp32")
        ids = torch.randint(0, cfg.vocab_size, (1, T), device=dev,
                            generator=torch.Generator(device=dev).manual_seed(10 + rank))
        labels = torch.cat([ids[:, 1:], torch.full((1, 1), -1, device=dev)], 1).int()
        for _ in range(2):
            trainer.train_step(ids, labels, T - 1)
        torch.cuda.synchronize()
        ep.check()
        reps = sorted(pl.replicated)
        for layer in model.layers:
            for p, full in ((layer.w_gu, full_gu), (layer.w_d, full_d)):
                rows = torch.stack([p.detach()[pl.slot_of(rank, e)] for e in reps]).contiguous()
                got = [torch.empty_like(rows) for _ in range(world)]
                dist.all_gather(got, rows)
                for other in got[1:]:
                    assert torch.equal(other, got[0])  # every copy took the same step
                assert not torch.equal(rows.cpu(), full[reps])  # and the step moved them
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


def test_replicated_experts_stay_identical_through_training():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_replica_train_worker, args=(2, _free_port(), errq), nprocs=2, join=True)
    assert errq.empty()


def _ep_dp_worker(rank, world, port, errq):
    """EP over blocks of world / 2 ranks, expert data parallel over the 2 blocks."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from spec_ep.integrations.ds_moe import make_groups
        from spec_ep.models.config import get_config
        from spec_ep.models.qwen3_moe import Qwen3MoeForCausalLM
        from spec_ep.parallel.ep import ExpertParallel
        from spec_ep.train import Trainer

        ep_size = world // 2
        ep_group, dp_group = make_groups(ep_size)
        assert dp_group is not None and dist.get_world_size(dp_group) == 2
        cfg = get_config("tiny", num_experts=8, top_k=2)
        T = 256
        ep = ExpertParallel(cfg.num_experts, cfg.top_k, cfg.hidden_size, max_tokens=T, group=ep_group, device=dev)
        torch.manual_seed(0)  # the same initial weights on every rank: replicas start equal
        model = Qwen3MoeForCausalLM(cfg, ep, device=dev)
        start = [p.detach().clone() for p in model.expert_parameters()]
        trainer = Trainer(model, lr=1e-2, expert_state="8bit", expert_dp_group=dp_group)
        assert trainer.expert_updater.fused_wgrad is None  # replicas need the summed gradient
        ids = torch.randint(0, cfg.vocab_size, (1, T), device=dev,
                            generator=torch.Generator(device=dev).manual_seed(10 + rank))
        labels = torch.cat([ids[:, 1:], torch.full((1, 1), -1, device=dev)], 1).int()
        losses = [float(trainer.train_step(ids, labels, T - 1)) for _ in range(3)]
        torch.cuda.synchronize()
        ep.check()
        assert all(x == x for x in losses)
        assert not trainer.expert_updater.pending
        for p, p0 in zip(model.expert_parameters(), start):
            got = [torch.empty_like(p) for _ in range(2)]
            dist.all_gather(got, p.detach().contiguous(), group=dp_group)
            assert torch.equal(got[0], got[1])  # the two replicas took the same steps
            assert not torch.equal(p.detach(), p0)  # and the steps moved them
        for p in model.dense_parameters():
            got = [torch.empty_like(p) for _ in range(world)]
            dist.all_gather(got, p.detach().contiguous())
            for other in got[1:]:
                assert torch.equal(other, got[0])
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception:
        import traceback

        errq.put((rank, traceback.format_exc()))
        raise


def test_expert_data_parallel_replicas_stay_identical():
    """EP x DP training (EP = 2 x DP = 2 on 4 GPUs, EP = 1 x DP = 2 on 2): the expert-DP
    gradient all-reduce runs asynchronously inside the backward and every replica of an
    expert takes the same update."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 4 if n >= 4 else 2
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.spawn(_ep_dp_worker, args=(world, _free_port(), errq), nprocs=world, join=True)
    assert errq.empty()
