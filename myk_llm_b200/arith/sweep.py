"""Arithmetic sweeps: run a grid (:mod:`myk_llm_b200.utils.sweep`) and tabulate accuracy
beyond the training lengths.

    python -m myk_llm_b200.arith.sweep configs/arith/sweeps/format-position.yaml
    python -m myk_llm_b200.arith.sweep configs/arith/sweeps/format-position.yaml --report
"""

from __future__ import annotations

import argparse
from pathlib import Path

import yaml

from ..utils.sweep import group_seeds, load_results, plan, run_all

METRICS = ("accuracy", "accuracy_late", "fillers_accuracy", "fillers_accuracy_late")


def extra_digits(result: dict, metric: str = "accuracy", threshold: float = 0.5) -> int:
    """Lengths past training at >= threshold, counted up from train_digits + 1."""
    n, d = 0, result["train_digits"] + 1
    while result[metric].get(str(d), 0.0) >= threshold:
        n, d = n + 1, d + 1
    return n


def report(sweep_dir: Path, metric: str = "accuracy") -> str:
    """Markdown table per task: seeds averaged, ``+digits`` (mean lengths past training at
    >= 50%), ``spread`` (largest seed gap at any length), accuracy at each longer length."""
    results = [{**r, "accuracy": r[metric]} for r in load_results(sweep_dir) if metric in r]
    if not results:
        return f"(no finished runs with {metric})"
    lines = []
    for task in sorted({r["run_name"].split("-")[0] for r in results}):
        grp = [r for r in results if r["run_name"].split("-")[0] == task]
        td = grp[0]["train_digits"]
        lengths = sorted({int(d) for r in grp for d in r["accuracy"]} - set(range(td + 1)))
        while lengths and all(r["accuracy"].get(str(lengths[-1]), 0.0) == 0.0 for r in grp):
            lengths.pop()
        lines += [f"\n### {task}, {metric} (trained on 1-{td} digits)\n",
                  "| run | seeds | in-dist | +digits | spread | " + " | ".join(map(str, lengths)) + " | min |",
                  "|---|---|---|---|---|" + "---|" * len(lengths) + "---|"]
        rows = []
        for name, runs in group_seeds(grp).items():
            acc = {d: [r["accuracy"].get(str(d), 0.0) for r in runs] for d in lengths}
            spread = max((max(v) - min(v) for v in acc.values()), default=0.0)
            plus = sum(extra_digits(r) for r in runs) / len(runs)
            tr = [str(d) for d in range(1, td + 1)]
            ind = 100 * sum(sum(r["accuracy"].get(d, 0.0) for d in tr if d in r["accuracy"]) /
                            max(1, sum(d in r["accuracy"] for d in tr)) for r in runs) / len(runs)
            mins = sum(r["train_minutes"] for r in runs) / len(runs)
            cells = " | ".join(f"{100 * sum(v) / len(v):.0f}" for v in acc.values())
            rows.append((-plus, f"| {name} | {len(runs)} | {ind:.1f} | {plus:.1f} | {100 * spread:.0f} | {cells} | "
                                f"{mins:.1f} |"))
        lines += [r for _, r in sorted(rows)]
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep")
    ap.add_argument("--report", action="store_true")
    ap.add_argument("--metric", choices=METRICS, default=None)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--output-dir", default="runs/arith")
    args = ap.parse_args(argv)
    sweep = yaml.safe_load(Path(args.sweep).read_text(encoding="utf-8"))
    sweep_dir = Path(args.output_dir) / sweep["name"]
    if not args.report:
        run_all(plan(sweep), sweep_dir, "myk_llm_b200.arith.train", args.dry_run)
    metrics = [args.metric] if args.metric else list(METRICS)
    table = "\n".join(t for t in (report(sweep_dir, m) for m in metrics) if not t.startswith("(no finished"))
    table = table or "(no finished runs)"
    print(table)
    if sweep_dir.exists():
        (sweep_dir / "summary.md").write_text(table + "\n", encoding="utf-8")


if __name__ == "__main__":
    main()
