"""Device-side stage timeline (spec_ep.utils.trace)."""
import pytest
import torch


@pytest.mark.gpu
def test_timeline_spans_pair_and_order():
    from spec_ep.utils.profile import stage
    from spec_ep.utils.trace import DeviceTimeline, enable_stage_timeline

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    tl = DeviceTimeline(capacity=64, device=dev)
    a = torch.randn(2048, 2048, device=dev)
    enable_stage_timeline(tl)
    try:
        for _ in range(3):
            with stage("matmul"):
                a = (a @ a).tanh()
        with tl.span("outer"):
            with stage("inner"):
                a = a * 2
    finally:
        enable_stage_timeline(None)
    ev = tl.events()
    assert [n for n, _ in ev][:2] == ["matmul:begin", "matmul:end"]
    ts = [t for _, t in ev]
    assert ts == sorted(ts)  # one stream: stamps in launch order
    d = tl.durations()
    assert d["matmul"]["count"] == 3 and d["matmul"]["total_us"] > 0
    assert d["outer"]["total_us"] >= d["inner"]["total_us"]
    # wrap-around keeps the newest entries in order
    small = DeviceTimeline(capacity=4, device=dev)
    for i in range(6):
        small.mark(f"m{i}")
    assert [n for n, _ in small.events()] == ["m2", "m3", "m4", "m5"]
