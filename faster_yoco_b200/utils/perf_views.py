"""SVG performance views rendered from JSON with no plotting library (docs/performance-views/render.py of the
reference draws the same three views with matplotlib, which this image does not have).

    python -m faster_yoco_b200.utils.perf_views DATA_DIR OUT_DIR

Inputs in DATA_DIR (any subset):
* ``history.json``: ``[{"label": str, "ms_per_update": float, "n_gpus": int}, ...]`` -> ``history.svg`` (bars)
* ``time-budget.json``: ``{"title": str, "phases": [[name, ms], ...]}`` -> ``time-budget.svg`` (stacked bar + legend)
* ``validation.json``: ``{"arms": {arm: {"updates": [...], "loss": [...]}}}`` -> ``validation.svg`` (lines)
"""
from __future__ import annotations

import json
import os
import sys
from html import escape
from typing import Dict, List, Sequence, Tuple

PALETTE = ["#4e79a7", "#f28e2b", "#e15759", "#76b7b2", "#59a14f", "#edc948", "#b07aa1", "#ff9da7", "#9c755f",
           "#bab0ac"]


def _svg(w: int, h: int, body: List[str]) -> str:
    return (f'<svg xmlns="http://www.w3.org/2000/svg" width="{w}" height="{h}" viewBox="0 0 {w} {h}" '
            f'font-family="sans-serif" font-size="12">\n<rect width="{w}" height="{h}" fill="white"/>\n'
            + "\n".join(body) + "\n</svg>\n")


def bars(items: Sequence[Tuple[str, float]], title: str, unit: str, width: int = 760) -> str:
    row, left, top = 26, 260, 40
    h = top + row * len(items) + 30
    vmax = max((v for _, v in items), default=1.0) or 1.0
    span = width - left - 90
    body = [f'<text x="10" y="22" font-size="15" font-weight="bold">{escape(title)}</text>']
    for i, (label, v) in enumerate(items):
        y = top + i * row
        bw = span * v / vmax
        body.append(f'<text x="{left - 8}" y="{y + 15}" text-anchor="end">{escape(label)}</text>')
        body.append(f'<rect x="{left}" y="{y + 3}" width="{bw:.1f}" height="{row - 8}" fill="{PALETTE[0]}"/>')
        body.append(f'<text x="{left + bw + 6:.1f}" y="{y + 15}">{v:.1f} {escape(unit)}</text>')
    return _svg(width, h, body)


def stacked(phases: Sequence[Tuple[str, float]], title: str, width: int = 760) -> str:
    total = sum(v for _, v in phases) or 1.0
    left, top, barh = 20, 40, 36
    span = width - 2 * left
    body = [f'<text x="10" y="22" font-size="15" font-weight="bold">{escape(title)} ({total:.1f} ms)</text>']
    x = left
    for i, (name, v) in enumerate(phases):
        w = span * v / total
        body.append(f'<rect x="{x:.1f}" y="{top}" width="{w:.1f}" height="{barh}" fill="{PALETTE[i % len(PALETTE)]}"/>')
        x += w
    for i, (name, v) in enumerate(phases):
        y = top + barh + 24 + i * 20
        body.append(f'<rect x="{left}" y="{y - 10}" width="12" height="12" fill="{PALETTE[i % len(PALETTE)]}"/>')
        body.append(f'<text x="{left + 18}" y="{y}">{escape(name)}: {v:.2f} ms ({100 * v / total:.1f}%)</text>')
    return _svg(width, top + barh + 40 + 20 * len(phases), body)


def lines(series: Dict[str, Tuple[Sequence[float], Sequence[float]]], title: str, xlabel: str, ylabel: str,
          width: int = 760, height: int = 420) -> str:
    left, right, top, bottom = 70, 140, 40, 50
    xs = [x for s in series.values() for x in s[0]] or [0, 1]
    ys = [y for s in series.values() for y in s[1]] or [0, 1]
    x0, x1 = min(xs), max(xs) if max(xs) > min(xs) else min(xs) + 1
    y0, y1 = min(ys), max(ys) if max(ys) > min(ys) else min(ys) + 1
    pw, ph = width - left - right, height - top - bottom
    X = lambda x: left + pw * (x - x0) / (x1 - x0)
    Y = lambda y: top + ph * (1 - (y - y0) / (y1 - y0))
    body = [f'<text x="10" y="22" font-size="15" font-weight="bold">{escape(title)}</text>',
            f'<rect x="{left}" y="{top}" width="{pw}" height="{ph}" fill="none" stroke="#999"/>',
            f'<text x="{left + pw / 2}" y="{height - 12}" text-anchor="middle">{escape(xlabel)}</text>',
            f'<text x="16" y="{top + ph / 2}" transform="rotate(-90 16 {top + ph / 2})" '
            f'text-anchor="middle">{escape(ylabel)}</text>']
    for k in range(5):
        yv = y0 + (y1 - y0) * k / 4
        xv = x0 + (x1 - x0) * k / 4
        body.append(f'<text x="{left - 6}" y="{Y(yv) + 4:.1f}" text-anchor="end">{yv:.3g}</text>')
        body.append(f'<text x="{X(xv):.1f}" y="{top + ph + 16}" text-anchor="middle">{xv:.4g}</text>')
    for i, (name, (sx, sy)) in enumerate(series.items()):
        c = PALETTE[i % len(PALETTE)]
        pts = " ".join(f"{X(x):.1f},{Y(y):.1f}" for x, y in zip(sx, sy))
        body.append(f'<polyline points="{pts}" fill="none" stroke="{c}" stroke-width="1.6"/>')
        body.append(f'<text x="{left + pw + 10}" y="{top + 16 + 18 * i}" fill="{c}">{escape(name)}</text>')
    return _svg(width, height, body)


def render(data_dir: str, out_dir: str) -> List[str]:
    os.makedirs(out_dir, exist_ok=True)
    written = []
    p = os.path.join(data_dir, "history.json")
    if os.path.exists(p):
        hist = json.load(open(p))
        items = [(f'{h["label"]} ({h.get("n_gpus", 1)} GPU)', float(h["ms_per_update"])) for h in hist]
        written.append(_write(out_dir, "history.svg", bars(items, "ms per update (YOCO-3B, 2048 tokens/GPU)", "ms")))
    p = os.path.join(data_dir, "time-budget.json")
    if os.path.exists(p):
        tb = json.load(open(p))
        written.append(_write(out_dir, "time-budget.svg",
                              stacked([(n, float(v)) for n, v in tb["phases"]], tb.get("title", "time budget"))))
    p = os.path.join(data_dir, "exchange.json")
    if os.path.exists(p):
        ex = json.load(open(p))
        written.append(_write(out_dir, "exchange.svg",
                              bars([(n, float(v)) for n, v in ex["bars"]], ex.get("title", "exchange"), "GB/s")))
    p = os.path.join(data_dir, "validation.json")
    if os.path.exists(p):
        v = json.load(open(p))
        series = {arm: (d["updates"], d["loss"]) for arm, d in v["arms"].items()}
        written.append(_write(out_dir, "validation.svg",
                              lines(series, "training loss (bits)", "update", "loss (bits)")))
    return written


def _write(out_dir: str, name: str, text: str) -> str:
    path = os.path.join(out_dir, name)
    with open(path, "w") as f:
        f.write(text)
    return path


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    for p in render(argv[0], argv[1] if len(argv) > 1 else argv[0]):
        print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
