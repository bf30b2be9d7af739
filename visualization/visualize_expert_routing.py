"""Plot expert popularity across experts and GPUs from routing dumps.

Reads one or more ``experts_rank{r}.pt`` files (each ``[L, T, K]`` int16 expert ids, as
written by ``spec_ep.utils.profile.RoutingRecorder``), concatenated along tokens. Per
layer, four bar panels: tokens per expert, the same sorted high to low, tokens per GPU
(contiguous blocks of ``num_experts // num_gpus`` experts, or a placement JSON), and
that sorted; a dashed line marks the balanced mean. Saves ``<first file>.png`` next to
the first input and a CSV of the histograms (reference:
visualization/visualize_expert_routing.py:38-92).

Rendering uses matplotlib's headless Agg backend when installed, otherwise PIL.

    python visualization/visualize_expert_routing.py logs/run/experts_rank*.pt --num_experts 128 --num_gpus 8
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def histograms(route: torch.Tensor, num_experts: int, num_gpus: int, owner=None, placement=None, sources=None):
    """Per layer: (tokens per expert [E], tokens per GPU [G]).

    GPU load follows ``placement`` (a ``spec_ep.parallel.placement.Placement``) when given:
    with ``sources`` (the source rank of every token, e.g. one dump file per rank) each
    token's copy goes where that source's routing tables send it, so replicated experts
    count on the rank that serves them; without sources, replicated experts' rows split
    evenly over the source ranks. Otherwise ``owner`` (expert -> rank) or contiguous
    blocks of ``num_experts // num_gpus`` experts.
    """
    out = []
    owner_t = torch.tensor(owner) if owner is not None else torch.arange(num_experts) // (num_experts // num_gpus)
    tables = None
    if placement is not None and sources is not None:
        tables = torch.stack([placement.tables(r)[0].long() for r in range(placement.world)])  # [W, E]
    for l in range(route.shape[0]):
        ids = route[l].reshape(-1).long()
        e = torch.bincount(ids, minlength=num_experts)
        if tables is not None:
            src = sources.long().repeat_interleave(route.shape[2])
            g = torch.bincount(tables[src, ids], minlength=num_gpus)
        elif placement is not None:
            g = placement.expected_rows(e).round().long()
        else:
            g = torch.zeros(num_gpus, dtype=torch.long).index_add_(0, owner_t, e)
        out.append((e, g))
    return out


def _draw_pil(hists, path, title):
    from PIL import Image, ImageDraw

    L = len(hists)
    W, row_h, pad = 1600, 140, 30
    widths = [0.4, 0.4, 0.1, 0.1]
    img = Image.new("RGB", (W, pad + L * row_h + 10), "white")
    d = ImageDraw.Draw(img)
    d.text((10, 8), title, fill="black")
    cols = ["tokens per expert", "experts, sorted", "tokens per GPU", "GPUs, sorted"]
    x0 = 10
    xs = []
    for w in widths:
        xs.append((x0, x0 + int(w * (W - 60))))
        x0 += int(w * (W - 60)) + 10
    for c, (a, b) in enumerate(xs):
        d.text((a, pad - 14), cols[c], fill="black")
    for l, (e, g) in enumerate(hists):
        y_top = pad + l * row_h + 5
        y_bot = y_top + row_h - 15
        panels = [e, e.sort(descending=True).values, g, g.sort(descending=True).values]
        for c, h in enumerate(panels):
            a, b = xs[c]
            top = max(int(panels[0 if c < 2 else 2].max()), 1)
            n = h.numel()
            bw = (b - a) / n
            for i, v in enumerate(h.tolist()):
                hh = int((y_bot - y_top) * v / top)
                d.rectangle([a + i * bw, y_bot - hh, a + (i + 1) * bw - (1 if bw > 3 else 0), y_bot], fill=(31, 119, 180))
            mean = float(h.float().mean())
            ym = y_bot - int((y_bot - y_top) * mean / top)
            for xx in range(a, b, 6):
                d.line([xx, ym, xx + 3, ym], fill=(214, 39, 40))
            d.text((a, y_top), f"L{l}", fill="black")
    img.save(path)


def _draw_mpl(hists, path, title):
    import matplotlib

    matplotlib.use("Agg")
    import matplotlib.pyplot as plt

    L = len(hists)
    fig, axes = plt.subplots(L, 4, figsize=(20, 1.8 * L), squeeze=False,
                             gridspec_kw={"width_ratios": [4, 4, 1.5, 1.5]})
    for l, (e, g) in enumerate(hists):
        panels = [e, e.sort(descending=True).values, g, g.sort(descending=True).values]
        for c, h in enumerate(panels):
            ax = axes[l, c]
            ax.bar(range(h.numel()), h, width=1.0 if c < 2 else 0.8)
            ax.axhline(h.float().mean(), color="red", lw=0.8, ls="--")
            ax.tick_params(labelsize=6)
        axes[l, 0].set_ylabel(f"L{l}", fontsize=8, rotation=0, labelpad=14, va="center")
    for c, t in enumerate(["tokens per expert", "experts, sorted", "tokens per GPU", "GPUs, sorted"]):
        axes[0, c].set_title(t, fontsize=9)
    fig.suptitle(title, y=1.0)
    fig.tight_layout()
    fig.savefig(path, dpi=120)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("files", nargs="+", type=Path, help="experts_rank*.pt, each [L, T, K]")
    ap.add_argument("--num_experts", type=int, default=128)
    ap.add_argument("--num_gpus", type=int, default=8)
    ap.add_argument("--placement", type=Path, default=None, help="placement JSON (Placement.to_dict)")
    args = ap.parse_args(argv)
    dumps = [torch.load(f).long() for f in args.files]
    route = torch.cat(dumps, dim=1)
    placement = sources = None
    if args.placement:
        from spec_ep.parallel.placement import Placement

        placement = Placement.from_dict(json.loads(args.placement.read_text()))
        if len(dumps) == placement.world:  # one dump per source rank: exact serving ranks
            sources = torch.cat([torch.full((d.shape[1],), r) for r, d in enumerate(dumps)])
    hists = histograms(route, args.num_experts, args.num_gpus, placement=placement, sources=sources)
    title = (f"Routing distribution ({len(args.files)} rank file(s), {route.shape[1]} tokens, "
             f"top-{route.shape[2]}); dashed = balanced level")
    out = args.files[0].with_suffix(".png")
    try:
        _draw_mpl(hists, out, title)
    except ImportError:
        _draw_pil(hists, out, title)
    csv = args.files[0].with_suffix(".csv")
    with open(csv, "w") as f:
        f.write("layer,kind,index,tokens\n")
        for l, (e, g) in enumerate(hists):
            f.writelines(f"{l},expert,{i},{v}\n" for i, v in enumerate(e.tolist()))
            f.writelines(f"{l},gpu,{i},{v}\n" for i, v in enumerate(g.tolist()))
    print(f"saved {out} and {csv}")
    return out


if __name__ == "__main__":
    main()
