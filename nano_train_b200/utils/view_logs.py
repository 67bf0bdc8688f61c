"""View training logs.

    python -m nano_train_b200.utils.view_logs --logdir outputs [--port 6006] [--host localhost] [--html out.html]

With TensorBoard installed this starts its server on ``--logdir`` (what the reference's
``scripts/view_logs.py`` does through its ``start_tensorboard.sh``); it serves until interrupted.
``--html`` instead renders every run's scalars into one HTML page of SVG charts (one chart per tag, one
line per run) that any browser opens offline; that is also what happens without TensorBoard. The
scalars come from TensorBoard event files (when the package is there) and from the
``<log_dir>/<run>/metrics.jsonl`` files the Trainer writes when it is not (one ``{"tag", "value",
"step"}`` object per line).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
from collections import defaultdict
from html import escape

from .svg_plot import Series, chart_svg


def read_jsonl_runs(logdir: str) -> dict:
    """{run: {tag: [(step, value), ...]}} from every ``metrics.jsonl`` under ``logdir``."""
    runs: dict = {}
    for root, _, files in os.walk(logdir):
        if "metrics.jsonl" not in files:
            continue
        run = os.path.relpath(root, logdir)
        tags = defaultdict(list)
        with open(os.path.join(root, "metrics.jsonl")) as f:
            for line in f:
                try:
                    rec = json.loads(line)
                    tags[str(rec["tag"])].append((int(rec["step"]), float(rec["value"])))
                except (ValueError, KeyError, TypeError):
                    continue  # a partly written last line
        runs[run] = {t: sorted(v) for t, v in tags.items()}
    return runs


def read_tfevent_runs(logdir: str) -> dict:
    """Same structure from TensorBoard event files (needs the tensorboard package)."""
    from tensorboard.backend.event_processing.event_accumulator import EventAccumulator

    runs: dict = {}
    for root, _, files in os.walk(logdir):
        if not any(f.startswith("events.out.tfevents") for f in files):
            continue
        ea = EventAccumulator(root, size_guidance={"scalars": 0})
        ea.Reload()
        tags = {t: sorted((e.step, float(e.value)) for e in ea.Scalars(t)) for t in ea.Tags().get("scalars", [])}
        if tags:
            runs[os.path.relpath(root, logdir)] = tags
    return runs


def render_html(runs: dict, title: str = "training logs") -> str:
    tags = sorted({t for r in runs.values() for t in r})
    parts = [f"<!doctype html><html><head><meta charset='utf-8'><title>{escape(title)}</title></head>",
             f"<body style='font-family:sans-serif'><h2>{escape(title)}</h2>",
             f"<p>{len(runs)} run(s): {escape(', '.join(sorted(runs)))}</p>"]
    for tag in tags:
        series = [Series(run, [s for s, _ in r[tag]], [v for _, v in r[tag]], kind="line" if len(r[tag]) > 1
                         else "points") for run, r in sorted(runs.items()) if tag in r]
        try:
            parts.append(chart_svg(None, series, title=tag, xlabel="step", ylabel=tag.split("/")[-1], logx=False,
                                   logy=False, width=720, height=320))
        except ValueError:
            continue  # nothing finite to draw
    parts.append("</body></html>")
    return "\n".join(parts)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="View nano_train_b200 training logs")
    ap.add_argument("--logdir", default="outputs")
    ap.add_argument("--port", default="6006")
    ap.add_argument("--host", default="localhost")
    ap.add_argument("--html", default=None, help="write the HTML page here (default: <logdir>/metrics.html)")
    a = ap.parse_args(argv)
    try:
        import tensorboard  # noqa: F401

        have_tb = True
    except ImportError:
        have_tb = False
    if have_tb and a.html is None:
        return subprocess.call([sys.executable, "-m", "tensorboard.main", "--logdir", a.logdir, "--port", a.port,
                                "--host", a.host])
    runs = read_jsonl_runs(a.logdir)
    if have_tb:
        for run, tags in read_tfevent_runs(a.logdir).items():
            runs.setdefault(run, tags)
    if not runs:
        print(f"no metrics.jsonl under {a.logdir}", file=sys.stderr)
        return 1
    out = a.html or os.path.join(a.logdir, "metrics.html")
    with open(out, "w") as f:
        f.write(render_html(runs, title=f"training logs: {a.logdir}"))
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
