"""Training launcher loop (spec_ep.run) on CPU: batches, metrics, checkpoints, resume."""
import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spec_ep.run import TokenBatches, train_loop


class _TinyTrainer:
    """Stands in for spec_ep.train.Trainer: embedding + linear head, SGD."""

    def __init__(self, vocab):
        torch.manual_seed(0)
        self.model = torch.nn.Sequential(torch.nn.Embedding(vocab, 16), torch.nn.Linear(16, vocab))
        self.opt = torch.optim.SGD(self.model.parameters(), lr=0.5)

    def train_step_from_host(self, ids, labels, num_valid=None):
        logits = self.model(ids.view(-1))
        loss = torch.nn.functional.cross_entropy(logits, labels.view(-1).long(), ignore_index=-1)
        self.opt.zero_grad()
        loss.backward()
        self.opt.step()
        return float(loss)


def test_batches_are_deterministic_and_disjoint(tmp_path):
    a = TokenBatches(100, 16, 2, rank=1, world=4, seed=3)
    b = TokenBatches(100, 16, 2, rank=1, world=4, seed=3)
    assert torch.equal(a.get(7)[0], b.get(7)[0]) and not torch.equal(a.get(7)[0], a.get(8)[0])
    assert (a.get(0)[1][:, -1] == -1).all()
    toks = np.arange(10_000, dtype=np.uint32) % 97
    path = tmp_path / "tokens.bin"
    toks.tofile(path)
    n = 16
    for step in range(3):
        for r in range(4):
            ids, lab = TokenBatches(97, 8, 2, r, 4, token_file=str(path)).get(step)
            assert torch.equal(lab.view(-1)[:-1].long(), ids.view(-1)[1:])  # next-token labels
            w = step * 4 + r  # window of (step, rank): disjoint across ranks and steps
            assert torch.equal(ids.view(-1), torch.from_numpy(toks[w * n:(w + 1) * n].astype(np.int64)))


def test_train_loop_metrics_checkpoints_and_resume(tmp_path):
    saved = []
    printed = []
    tr = _TinyTrainer(50)
    batches = TokenBatches(50, 8, 4, 0, 1, seed=1)
    recs = train_loop(tr, batches, 6, 0, str(tmp_path), ckpt_every=2,
                      save_fn=lambda p, s: saved.append((os.path.basename(p), s)), print_fn=printed.append)
    assert [r["step"] for r in recs] == list(range(6))
    assert saved == [("step_2", 2), ("step_4", 4), ("step_6", 6)]
    lines = [json.loads(x) for x in open(tmp_path / "metrics_rank0.jsonl")]
    assert len(lines) == 6 and all(x["ms"] > 0 and x["tokens_per_s_rank"] > 0 for x in lines)
    assert len(printed) == 6 and "tokens_per_s" in json.loads(printed[0])
    # resuming at step 4 replays exactly the batches an uninterrupted run would see
    more = train_loop(_TinyTrainer(50), TokenBatches(50, 8, 4, 0, 1, seed=1), 6, 4, None, print_fn=None)
    assert [r["step"] for r in more] == [4, 5]


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, port, out):
    from spec_ep.utils.heartbeat import Heartbeat

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        printed = []
        recs = train_loop(_TinyTrainer(40), TokenBatches(40, 8, 2, rank, 2, seed=5), 3, 0, None,
                          print_fn=printed.append)
        # resumed at step 3 with a heartbeat: arrivals count from the resume point
        hb = Heartbeat.from_default_group(timeout_s=30.0)
        more = train_loop(_TinyTrainer(40), TokenBatches(40, 8, 2, rank, 2, seed=5), 5, 3, None,
                          print_fn=None, heartbeat=hb)
        out[rank] = (len(recs), len(printed), [r["step"] for r in more], hb.arrived)
    finally:
        dist.destroy_process_group()


def test_train_loop_two_gloo_ranks():
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(_free_port(), out), nprocs=2, join=True)
    assert out[0] == (3, 3, [3, 4], 2) and out[1] == (3, 0, [3, 4], 2)  # only rank 0 prints the job line


@pytest.mark.gpu
def test_launcher_trains_checkpoints_and_resumes_tiny_model(tmp_path, capsys):
    from spec_ep.run import main

    log = str(tmp_path / "run")
    main(["--model", "tiny", "--seq", "256", "--steps", "4", "--log-dir", log, "--ckpt-every", "2", "--ep-stats"])
    lines = [json.loads(x) for x in open(os.path.join(log, "metrics_rank0.jsonl"))]
    assert [x["step"] for x in lines] == [0, 1, 2, 3]
    assert all(x["loss"] == x["loss"] and x["tokens"] > 0 for x in lines)
    assert lines[0]["remote_rows_per_token"] == 0.0 and lines[0]["naive_rows_per_token"] == 0.0  # one GPU
    assert os.path.exists(os.path.join(log, "step_2", "meta.json"))
    main(["--model", "tiny", "--seq", "256", "--steps", "4", "--log-dir", log + "_resumed", "--resume",
          os.path.join(log, "step_2")])
    resumed = [json.loads(x) for x in open(os.path.join(log + "_resumed", "metrics_rank0.jsonl"))]
    assert [x["step"] for x in resumed] == [2, 3]
    # same weights, optimizer state and batches: the resumed steps repeat the original losses
    for a, b in zip(resumed, lines[2:]):
        assert abs(a["loss"] - b["loss"]) <= 1e-3 * abs(b["loss"]), (a["loss"], b["loss"])


def test_train_loop_records_stage_times_from_a_timeline():
    """The loop turns the stage timeline on around each step only and records its
    per-stage means (a stand-in timeline: the device one is covered by the GPU tests)."""
    from spec_ep.utils.trace import active_timeline

    class _Timeline:
        def __init__(self):
            self.resets, self.seen = 0, []

        def reset(self):
            self.resets += 1

        def durations(self):
            return {"dispatch": {"count": 2, "total_us": 30.0, "mean_us": 15.0},
                    "combine": {"count": 2, "total_us": 10.0, "mean_us": 5.0}}

    class _Probe(_TinyTrainer):
        def train_step_from_host(self, ids, labels, num_valid=None):
            tl.seen.append(active_timeline())
            return super().train_step_from_host(ids, labels, num_valid)

    tl = _Timeline()
    recs = train_loop(_Probe(30), TokenBatches(30, 8, 2, 0, 1, seed=2), 3, 0, None, print_fn=None, timeline=tl)
    assert tl.resets == 3 and tl.seen == [tl, tl, tl] and active_timeline() is None
    assert recs[0]["stage_us"] == {"dispatch": {"mean_us": 15.0, "count": 2}, "combine": {"mean_us": 5.0, "count": 2}}
