"""Arithmetic sweeps: run a grid (:mod:`myk_llm_b200.utils.sweep`) and tabulate how far
accuracy reaches past the training lengths.

    python -m myk_llm_b200.arith.sweep configs/arith/sweeps/format-position.yaml
    python -m myk_llm_b200.arith.sweep configs/arith/sweeps/format-position.yaml --report

One table per task (the run-name prefix before the first ``-``), one row per configuration
with its seeds averaged: the in-distribution accuracy, ``+digits`` (how many lengths past
training stay at >= 50%, counted upward from the first one past training, averaged over
seeds), ``spread`` (the largest gap between seeds at any length), the accuracy at each
longer length, and the training minutes.  The report layout follows the reference's
``src/myk_llm/arith/sweep.py``.
"""

from __future__ import annotations

import argparse
from pathlib import Path
from statistics import mean

import yaml

from ..utils.sweep import group_seeds, load_results, plan, run_all

METRICS = ("accuracy", "accuracy_late", "fillers_accuracy", "fillers_accuracy_late")


def extra_digits(result: dict, metric: str = "accuracy", threshold: float = 0.5) -> int:
    """Consecutive lengths from ``train_digits + 1`` upward with accuracy >= threshold."""
    acc, d = result[metric], result["train_digits"] + 1
    while acc.get(str(d), 0.0) >= threshold:
        d += 1
    return d - result["train_digits"] - 1


def _longer_lengths(runs: list[dict], train_digits: int) -> list[int]:
    """Lengths past training, without trailing ones where every run scores zero."""
    lengths = sorted({int(d) for r in runs for d in r["accuracy"] if int(d) > train_digits})
    while lengths and not any(r["accuracy"].get(str(lengths[-1]), 0.0) for r in runs):
        lengths.pop()
    return lengths


def _row(name: str, runs: list[dict], lengths: list[int], train_digits: int) -> tuple[float, str]:
    per_len = {d: [r["accuracy"].get(str(d), 0.0) for r in runs] for d in lengths}
    spread = max((max(v) - min(v) for v in per_len.values()), default=0.0)
    plus = mean(extra_digits(r) for r in runs)
    inside = []
    for r in runs:
        have = [r["accuracy"][str(d)] for d in range(1, train_digits + 1) if str(d) in r["accuracy"]]
        inside.append(sum(have) / max(1, len(have)))
    cells = [name, str(len(runs)), f"{100 * mean(inside):.1f}", f"{plus:.1f}", f"{100 * spread:.0f}",
             *[f"{100 * mean(v):.0f}" for v in per_len.values()], f"{mean(r['train_minutes'] for r in runs):.1f}"]
    return -plus, "| " + " | ".join(cells) + " |"


def report(sweep_dir: Path, metric: str = "accuracy") -> str:
    runs = [dict(r, accuracy=r[metric]) for r in load_results(sweep_dir) if metric in r]
    if not runs:
        return f"(no finished runs with {metric})"
    out: list[str] = []
    for task in sorted({r["run_name"].split("-")[0] for r in runs}):
        mine = [r for r in runs if r["run_name"].split("-")[0] == task]
        td = mine[0]["train_digits"]
        lengths = _longer_lengths(mine, td)
        out += [f"\n### {task}, {metric} (trained on 1-{td} digits)\n",
                "| run | seeds | in-dist | +digits | spread | " + " | ".join(map(str, lengths)) + " | min |",
                "|---|---|---|---|---|" + "---|" * len(lengths) + "---|"]
        rows = [_row(name, group, lengths, td) for name, group in group_seeds(mine).items()]
        out += [text for _, text in sorted(rows)]
    return "\n".join(out)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep")
    ap.add_argument("--report", action="store_true")
    ap.add_argument("--metric", choices=METRICS, default=None)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--output-dir", default="runs/arith")
    args = ap.parse_args(argv)
    spec = yaml.safe_load(Path(args.sweep).read_text(encoding="utf-8"))
    sweep_dir = Path(args.output_dir) / spec["name"]
    if not args.report:
        run_all(plan(spec), sweep_dir, "myk_llm_b200.arith.train", args.dry_run)
    tables = [report(sweep_dir, m) for m in ([args.metric] if args.metric else METRICS)]
    text = "\n".join(t for t in tables if not t.startswith("(no finished")) or "(no finished runs)"
    print(text)
    if sweep_dir.exists():
        (sweep_dir / "summary.md").write_text(text + "\n", encoding="utf-8")


if __name__ == "__main__":
    main()
