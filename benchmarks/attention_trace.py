"""Pipeline trace of the two-tile tcgen05 attention forward (CTA 0, SM clock cycles).

Runs the Qwen3-30B-A3B attention shape (4096 tokens, 32 / 4 heads) with the kernel's
trace hook and prints, per tile, the median over steady-state key blocks of:
softmax (S ready -> P computed), publish, P ready -> MMA warp awake, P V issue, P V
issue -> done, next S issue -> S ready at the softmax, and the per-block period.

    python benchmarks/attention_trace.py
"""
import os
import statistics as st
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    from spec_ep.ops.attention import attention_fwd

    T, Hq, Hkv = 4096, 32, 4
    q = torch.randn(T, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    for _ in range(3):
        attention_fwd(q, k, v, two_tile=True)
    tr = torch.zeros(4, 64, 4, dtype=torch.int64, device="cuda")
    attention_fwd(q, k, v, two_tile=True, trace=tr)
    torch.cuda.synchronize()
    t = tr.cpu()
    rng = range(2, 28)  # steady state of CTA 0 (31 / 32 key blocks)
    for tt in range(2):
        med = lambda xs: st.median(xs)  # noqa: E731
        row = {
            "softmax": med([int(t[2 + tt, j, 1] - t[2 + tt, j, 0]) for j in rng]),
            "publish": med([int(t[2 + tt, j, 2] - t[2 + tt, j, 1]) for j in rng]),
            "P_ready_to_mma": med([int(t[tt, j, 0] - t[2 + tt, j, 2]) for j in rng]),
            "pv_issue": med([int(t[tt, j, 1] - t[tt, j, 0]) for j in rng]),
            "pv_issue_to_done": med([int(t[tt, j, 2] - t[tt, j, 1]) for j in rng]),
            "s_issue_to_softmax": med([int(t[2 + tt, j + 1, 0] - t[tt, j, 3]) for j in rng]),
            "period": med([int(t[2 + tt, j + 1, 0] - t[2 + tt, j, 0]) for j in rng]),
        }
        print(f"tile {'AB'[tt]} (cycles): {row}")


if __name__ == "__main__":
    import argparse

    argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter).parse_args()
    main()
