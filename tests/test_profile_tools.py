"""Host-side helpers of the step profiler (no GPU): kernel classification and the device
idle-gap report built from profiler events."""
import importlib.util
import os
from types import SimpleNamespace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _profile_step():
    spec = importlib.util.spec_from_file_location("profile_step", os.path.join(ROOT, "benchmarks", "profile_step.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ev(name, start, end, cuda=True):
    return SimpleNamespace(name=name, device_type="DeviceType.CUDA" if cuda else "DeviceType.CPU",
                           time_range=SimpleNamespace(start=start, end=end))


def test_kernel_classes():
    ps = _profile_step()
    assert ps.classify("void sepx::grouped_gemm_pair_kernel<256, 5, false, true, false, 2>(...)").startswith("expert")
    assert ps.classify("sepx::recv_gather_kernel(sepx::EpArgs, ...)").startswith("ep")
    assert ps.classify("cudnn_generated_fort_native_sdpa_sm100_flash_bprop_f16") == "attention bwd"
    assert ps.classify("void sepx::rmsnorm_bwd_kernel<8>(...)").startswith("norm")
    assert ps.classify("ncclDevKernel_AllReduce_Sum_bf16_RING_LL") == "collectives (NCCL)"
    assert ps.classify("something else entirely") == "other"


def test_gap_report_counts_idle_time_between_kernels():
    ps = _profile_step()
    events = [_ev("a", 0, 10), _ev("b", 12, 20), _ev("c", 15, 18),  # c overlaps b: no gap
              _ev("d", 150, 160), _ev("host", 20, 150, cuda=False), _ev("e", 1160, 1170)]
    prof = SimpleNamespace(events=lambda: events)
    text = ps.gaps(prof, top=3)
    # gaps: 2 us (a->b), 130 us (b->d), 1000 us (d->e)
    assert "idle 1.13 ms in 3 gaps" in text
    lines = text.splitlines()
    assert "| 1000.0 | d | e |" in lines and "| 130.0 | b | d |" in lines
    assert any(line.startswith("| 0-5 | 1 |") for line in lines)
