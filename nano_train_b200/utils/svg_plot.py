"""Minimal chart writer: line and point series on log or linear axes as standalone SVG.

The model-report plots (roofline with the model's operating points, decode batch sweep) and the
training-log viewer are plain text, so they need no plotting library and no graphics stack; any browser
renders them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional
from xml.sax.saxutils import escape

PALETTE = ("#1f77b4", "#d62728", "#2ca02c", "#9467bd", "#ff7f0e", "#8c564b", "#e377c2", "#17becf")


@dataclass
class Series:
    label: str
    xs: list
    ys: list
    kind: str = "line"          # "line" or "points"
    color: Optional[str] = None
    dashed: bool = False
    point_labels: list = field(default_factory=list)


def _ticks(lo: float, hi: float) -> list[float]:
    a, b = math.floor(math.log10(lo)), math.ceil(math.log10(hi))
    return [10.0 ** e for e in range(a, b + 1)]


def _fmt(v: float) -> str:
    if v > 0 and (v >= 1e6 or v < 1e-2):
        return f"1e{int(round(math.log10(v)))}"
    return f"{v:.6g}"


def _lin_ticks(lo: float, hi: float, n: int = 6) -> list[float]:
    """At most n + 2 round ticks in [lo, hi] (a bounded count: no loop that depends on float steps)."""
    span = hi - lo
    if not (span > 0 and math.isfinite(span)):
        return [lo]
    step = 10 ** math.floor(math.log10(span / n))
    for m in (1, 2, 5, 10):
        if span / (step * m) <= n:
            step *= m
            break
    first = math.ceil(lo / step)
    return [t for t in ((first + i) * step for i in range(n + 2)) if t <= hi]


def loglog_svg(path: str, series: list[Series], *, title: str, xlabel: str, ylabel: str,
               width: int = 760, height: int = 480) -> str:
    """Write ``series`` on log-log axes to ``path``; returns the path. Non-positive values are skipped."""
    return chart_svg(path, series, title=title, xlabel=xlabel, ylabel=ylabel, width=width, height=height)


def chart_svg(path: Optional[str], series: list[Series], *, title: str, xlabel: str, ylabel: str,
              logx: bool = True, logy: bool = True, width: int = 760, height: int = 480) -> str:
    """Chart of ``series`` (log or linear axes). Written to ``path`` when given; returns the SVG text
    if ``path`` is None, else the path. On a log axis non-positive values are skipped."""
    ok = lambda x, y: (x > 0 or not logx) and (y > 0 or not logy) and math.isfinite(x) and math.isfinite(y)  # noqa
    pts = [(x, y) for s in series for x, y in zip(s.xs, s.ys) if ok(x, y)]
    if not pts:
        raise ValueError("nothing to plot")
    x0, x1 = min(p[0] for p in pts), max(p[0] for p in pts)
    y0, y1 = min(p[1] for p in pts), max(p[1] for p in pts)
    if logx:
        x0, x1 = 10 ** math.floor(math.log10(x0)), 10 ** math.ceil(math.log10(x1 * 1.0001))
    elif x1 - x0 <= abs(x0) * 1e-9:
        x0, x1 = x0 - max(abs(x0) * 0.05, 1.0), x1 + max(abs(x1) * 0.05, 1.0)
    if logy:
        y0, y1 = 10 ** math.floor(math.log10(y0)), 10 ** math.ceil(math.log10(y1 * 1.0001))
    else:
        # a flat or nearly flat series (relative to its magnitude) gets a visible band around it
        pad = (y1 - y0) * 0.05 if y1 - y0 > abs(y0) * 1e-9 else max(abs(y0) * 0.05, 1e-12)
        y0, y1 = y0 - pad, y1 + pad
    ml, mr, mt, mb = 72, 190, 40, 56
    pw, ph = width - ml - mr, height - mt - mb
    fx = (lambda v: math.log10(v)) if logx else (lambda v: v)
    fy = (lambda v: math.log10(v)) if logy else (lambda v: v)

    def sx(x):
        return ml + pw * (fx(x) - fx(x0)) / (fx(x1) - fx(x0))

    def sy(y):
        return mt + ph * (1 - (fy(y) - fy(y0)) / (fy(y1) - fy(y0)))

    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" font-family="sans-serif" '
           f'font-size="11">', f'<rect width="{width}" height="{height}" fill="white"/>',
           f'<text x="{ml + pw / 2}" y="22" text-anchor="middle" font-size="14">{escape(title)}</text>']
    for t in (_ticks(x0, x1) if logx else _lin_ticks(x0, x1)):
        if x0 <= t <= x1:
            out.append(f'<line x1="{sx(t):.1f}" y1="{mt}" x2="{sx(t):.1f}" y2="{mt + ph}" stroke="#ddd"/>')
            out.append(f'<text x="{sx(t):.1f}" y="{mt + ph + 16}" text-anchor="middle">{_fmt(t)}</text>')
    for t in (_ticks(y0, y1) if logy else _lin_ticks(y0, y1)):
        if y0 <= t <= y1:
            out.append(f'<line x1="{ml}" y1="{sy(t):.1f}" x2="{ml + pw}" y2="{sy(t):.1f}" stroke="#ddd"/>')
            out.append(f'<text x="{ml - 6}" y="{sy(t) + 4:.1f}" text-anchor="end">{_fmt(t)}</text>')
    out.append(f'<rect x="{ml}" y="{mt}" width="{pw}" height="{ph}" fill="none" stroke="#333"/>')
    out.append(f'<text x="{ml + pw / 2}" y="{height - 14}" text-anchor="middle">{escape(xlabel)}</text>')
    out.append(f'<text x="16" y="{mt + ph / 2}" text-anchor="middle" '
               f'transform="rotate(-90 16 {mt + ph / 2})">{escape(ylabel)}</text>')
    for i, s in enumerate(series):
        c = s.color or PALETTE[i % len(PALETTE)]
        xy = [(sx(x), sy(y)) for x, y in zip(s.xs, s.ys) if ok(x, y)]
        if s.kind == "line" and len(xy) > 1:
            d = " ".join(f"{x:.1f},{y:.1f}" for x, y in xy)
            dash = ' stroke-dasharray="6,4"' if s.dashed else ""
            out.append(f'<polyline points="{d}" fill="none" stroke="{c}" stroke-width="1.8"{dash}/>')
        else:
            for j, (x, y) in enumerate(xy):
                out.append(f'<circle cx="{x:.1f}" cy="{y:.1f}" r="4" fill="{c}"/>')
                if j < len(s.point_labels):
                    out.append(f'<text x="{x + 6:.1f}" y="{y - 6:.1f}" fill="{c}">{escape(s.point_labels[j])}</text>')
        ly = mt + 14 + 16 * i
        out.append(f'<rect x="{ml + pw + 12}" y="{ly - 9}" width="12" height="10" fill="{c}"/>')
        out.append(f'<text x="{ml + pw + 30}" y="{ly}">{escape(s.label)}</text>')
    out.append("</svg>")
    text = "\n".join(out) + "\n"
    if path is None:
        return text
    with open(path, "w") as f:
        f.write(text)
    return path
