"""Training engine: one step = forward, backward, gradient sync, optimizer.

* Expert weights are sharded over the EP group and updated *inside* the backward pass
  (the MoE layer hands each expert gradient to the optimizer the moment its wgrad GEMM
  is done), so a full-model expert gradient buffer never exists.
* Dense weights (attention, router, norms, embeddings) are replicated on every rank;
  their gradients are all-reduced (NCCL, bucketed) over the data-parallel group, which
  for pure EP is every rank.
* Expert replicas inside the EP group (a planned placement that copies hot experts to
  every rank) each see only the tokens routed to their copy; their gradients are summed
  over the EP group before the update, so every copy takes the same step.
* Expert replicas across DP groups (EP < world) are all-reduced over the replica group
  before their in-backward update. The all-reduce of a layer's expert gradients runs
  asynchronously on NCCL's stream while the backward of the next-lower layer computes;
  the update of those weights is applied one layer later (and the last ones after the
  backward), so the expert-DP traffic overlaps compute instead of blocking it. The fused
  wgrad + 8-bit AdamW epilogue is not used in that case: it never materialises the
  gradient, and the update needs the gradient summed over the replicas.
* Optimizer state precision is chosen per parameter group to fit the memory budget:
  fp32 master + moments where they fit, block-wise 8-bit moments otherwise.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .ops.optim import FusedAdamW


def choose_state_precision(expert_params: int, dense_params: int, budget_bytes: int,
                           activation_bytes: int) -> str:
    """Most precise expert optimizer state that fits next to weights and activations."""
    weights = 2 * (expert_params + dense_params)
    dense_state = 12 * dense_params
    for prec, per in (("fp32", 12), ("8bit", 2.25)):
        if weights + dense_state + per * expert_params + activation_bytes <= budget_bytes:
            return prec
    return "8bit"


class Trainer:
    def __init__(self, model, lr=3e-4, weight_decay=0.1, betas=(0.9, 0.95), expert_state="fp32",
                 dp_group=None, expert_dp_group=None, bucket_mb=256, fuse_expert_optimizer=None):
        self.model = model
        self.dense = model.dense_parameters()
        self.experts = model.expert_parameters()
        for p in self.experts:
            p._sepx_state_precision = expert_state
        self.opt = FusedAdamW(self.dense + self.experts, lr=lr, betas=betas, weight_decay=weight_decay,
                              state_precision="fp32")
        self.dp_group = dp_group
        self.expert_dp_group = expert_dp_group
        self.world = dist.get_world_size(dp_group) if dist.is_initialized() else 1
        self.expert_world = dist.get_world_size(expert_dp_group) if (dist.is_initialized() and expert_dp_group
                                                                      is not None) else 1
        self.bucket_bytes = bucket_mb << 20
        if fuse_expert_optimizer is None:  # the 8-bit fused epilogue is the faster path
            fuse_expert_optimizer = expert_state == "8bit"
        self.fuse_expert_optimizer = fuse_expert_optimizer
        self.expert_updater = _ExpertUpdater(self)
        model.set_grad_sink(self.expert_updater)
        self.budget_retries = 0  # forwards run again because a row budget overflowed
        self.buckets = _GradBuckets(self.dense, self.dp_group, self.bucket_bytes) if self.world > 1 else None

    def _sync_dense_grads(self):
        """Wait for the bucketed all-reduces started during backward (ranks > 1)."""
        if self.buckets is not None:
            self.buckets.finish()

    def _forward(self, input_ids, labels, num_valid):
        """The loss, with the MoE layers' receive buffers sized by row budgets (no host
        wait between layers). If some layer's rows outgrew its budget on any rank, the
        forward is discarded (nothing was updated yet) and run again with the grown
        budgets; the first step learns the budgets with exact sizes."""
        ep = getattr(self.model, "ep", None)
        if ep is None or not hasattr(ep, "run_pass"):
            return self.model(input_ids, labels, num_valid)
        calls = [0]

        def fwd():
            calls[0] += 1
            return self.model(input_ids, labels, num_valid)

        loss = ep.run_pass(fwd)
        self.budget_retries += calls[0] - 1
        return loss

    def train_step(self, input_ids, labels, num_valid=None):
        """One optimizer step on a device-resident batch; returns the (device) loss."""
        if self.buckets is not None:
            self.buckets.begin()
        loss = self._forward(input_ids, labels, num_valid)
        loss.backward()
        self.expert_updater.flush()
        self._sync_dense_grads()
        self.opt.step()
        return loss.detach()

    def train_step_from_host(self, input_ids_cpu, labels_cpu, num_valid=None):
        """End-to-end step: pinned host batch -> device, step, loss read back to the host."""
        dev = self.model.ep.device
        ids = input_ids_cpu.to(dev, non_blocking=True)
        lab = labels_cpu.to(dev, non_blocking=True)
        loss = self.train_step(ids, lab, num_valid)
        return float(loss.to("cpu"))


class _GradBuckets:
    """Dense-gradient averaging overlapped with the backward pass.

    Dense parameters are packed, in reverse registration order (roughly the order their
    gradients become ready), into flat buckets of about ``bucket_bytes``; each slot starts
    on a 16-byte boundary so the optimizer kernels can read it with vector loads. A
    post-accumulate-grad hook copies each gradient into its slot and frees it; when a
    bucket's last gradient lands, an asynchronous NCCL all-reduce (average) of the bucket
    starts on NCCL's stream while backward continues. ``finish`` makes the compute stream
    wait for every bucket and hands the reduced slots to the optimizer as ``.grad`` views.
    A parameter that got no gradient in a step contributes zeros. Every rank runs the same
    model, so buckets complete in the same order on every rank.
    """

    def __init__(self, params, group, bucket_bytes):
        self.group = group
        self.active = False
        # NCCL averages in the collective; other backends sum and scale afterwards
        self.avg = dist.get_backend(group) == "nccl"
        self.world = dist.get_world_size(group)
        self.buckets = []  # (flat buffer, [(param, offset)])
        self.where = {}
        cur, size = [], 0
        for p in reversed(params):
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= bucket_bytes:
                self._add(cur)
                cur, size = [], 0
        if cur:
            self._add(cur)
        for p in params:
            p.register_post_accumulate_grad_hook(self._hook)

    def _add(self, ps):
        dtype, dev = ps[0].dtype, ps[0].device
        align = max(1, 16 // ps[0].element_size())
        off, slots = 0, []
        for p in ps:
            if p.dtype != dtype:
                raise TypeError("a gradient bucket holds one dtype")
            slots.append((p, off))
            off += (p.numel() + align - 1) // align * align
        b = len(self.buckets)
        self.buckets.append((torch.zeros(off, dtype=dtype, device=dev), slots))
        for i, (p, _) in enumerate(slots):
            self.where[id(p)] = (b, i)

    def begin(self):
        self.active = True
        self.pending = [len(slots) for _, slots in self.buckets]
        self.seen = [[False] * len(slots) for _, slots in self.buckets]
        self.works = [None] * len(self.buckets)

    def _hook(self, p):
        if not self.active:  # backward outside a training step: leave .grad alone
            return
        b, i = self.where[id(p)]
        flat, slots = self.buckets[b]
        off = slots[i][1]
        flat[off:off + p.numel()].copy_(p.grad.reshape(-1))
        p.grad = None
        self.seen[b][i] = True
        self.pending[b] -= 1
        if self.pending[b] == 0:
            self._launch(b)

    def _launch(self, b):
        op = dist.ReduceOp.AVG if self.avg else dist.ReduceOp.SUM
        self.works[b] = dist.all_reduce(self.buckets[b][0], op=op, group=self.group, async_op=True)

    def finish(self):
        for b, (flat, slots) in enumerate(self.buckets):
            if self.works[b] is None:  # some parameter got no gradient this step
                for i, (p, off) in enumerate(slots):
                    if not self.seen[b][i]:
                        flat[off:off + p.numel()].zero_()
                self._launch(b)
        for b, (flat, slots) in enumerate(self.buckets):
            self.works[b].wait()
            if not self.avg:
                flat.mul_(1.0 / self.world)
            for p, off in slots:
                p.grad = flat[off:off + p.numel()].view_as(p)
        self.active = False


def replica_slots(placement, rank: int) -> list[int]:
    """For each replicated expert of the placement (expert-id order), its local slot on
    ``rank``, or -1 where ``rank`` holds no copy (partial replication)."""
    if placement is None or not placement.replicated:
        return []
    return [placement.slot_of(rank, e) if rank in placement.holders_of(e) else -1
            for e in sorted(placement.replicated)]


def sum_replica_grads(g: torch.Tensor, slots: list[int], group=None):
    """Sum the gradient rows of replicated experts (``g`` is ``[local slots, ...]``) over
    ``group`` in place: each copy's gradient covers only the tokens it served, the
    expert's gradient is their sum. Every rank of ``group`` calls it with one entry per
    replicated expert (-1: no copy here, contributes zeros)."""
    if not slots or not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return g
    held = [i for i, s in enumerate(slots) if s >= 0]
    rows = g.new_zeros((len(slots),) + tuple(g.shape[1:]))
    if held:
        at = torch.tensor(held, dtype=torch.long, device=g.device)
        src = torch.tensor([slots[i] for i in held], dtype=torch.long, device=g.device)
        rows.index_copy_(0, at, g.index_select(0, src))
    dist.all_reduce(rows, group=group)
    if held:
        g.index_copy_(0, src, rows.index_select(0, at))
    return g


class _ExpertUpdater:
    """Receives expert weight gradients inside the MoE backward.

    With fused updates (the default for 8-bit expert state without expert replicas) the
    weight-gradient GEMM applies AdamW in its epilogue and the gradient never reaches
    HBM: the 8-bit epilogue streams W and its codes through a TMA ring and is ~10-25%
    faster than the two-kernel path on the Qwen3-30B-A3B shapes. Otherwise (fp32 state,
    or replicas that need an all-reduce of the gradient first) the GEMM writes an fp32
    gradient and the streaming optimizer kernel applies it.
    """

    # gradients whose expert-DP all-reduce may still be in flight: one layer's two
    # weights, while the next-lower layer's backward computes
    depth = 2

    def __init__(self, trainer):
        self.t = trainer
        ep = getattr(trainer.model, "ep", None)
        self.rep_slots = replica_slots(getattr(ep, "placement", None), ep.rank) if ep is not None else []
        self.ep_group = ep.group if ep is not None else None
        use = trainer.fuse_expert_optimizer and trainer.expert_world == 1 and not self.rep_slots
        self.fused_wgrad = trainer.opt.fused_wgrad if use else None
        self.pending = []  # (param, grad, work) with the expert-DP all-reduce in flight

    def __call__(self, p, g):
        t = self.t
        if self.rep_slots:
            sum_replica_grads(g, self.rep_slots, self.ep_group)
        if t.expert_world > 1:
            # start the replica all-reduce now; apply the update once it is needed
            work = dist.all_reduce(g, group=t.expert_dp_group, async_op=True)
            self.pending.append((p, g, work))
            while len(self.pending) > self.depth:
                self._apply(*self.pending.pop(0))
            return
        t.opt.apply_now(p, g)

    def _apply(self, p, g, work):
        work.wait()  # the compute stream waits for NCCL's; the host does not block
        g.mul_(1.0 / self.t.expert_world)
        self.t.opt.apply_now(p, g)

    def flush(self):
        """Apply every update still waiting for its all-reduce (end of the backward)."""
        while self.pending:
            self._apply(*self.pending.pop(0))
