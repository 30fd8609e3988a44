"""A grid of pretraining runs (``python -m myk_llm_b200.train``) and their summary table.

Sweep files and resume rules are those of :mod:`myk_llm_b200.utils.sweep` (every
combination of the axes is one run; a run with a ``results.json`` is skipped).  After a
run reaches its last step, its final validation metrics, median throughput (first 10 % of
records dropped as warm-up) and parameter counts go to ``<sweep_dir>/<run>/results.json``.
The report groups seeds (``-s<k>`` suffixes) and sorts by mean bits per byte::

    python -m myk_llm_b200.train.sweep_train configs/experiments/sweeps/ngram.yaml
    python -m myk_llm_b200.train.sweep_train configs/experiments/sweeps/ngram.yaml --report

(The reference's ``scripts/sweep_train.py``.)
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np
import yaml

from ..utils.sweep import group_seeds, load_results, plan, run_all


def summarize(run_dir: Path) -> dict | None:
    """Final validation metrics, throughput and parameter counts of a run, or None when it
    never evaluated."""
    path = run_dir / "metrics.jsonl"
    if not path.exists():
        return None
    recs = [json.loads(line) for line in path.read_text().splitlines() if line.strip()]
    evals = [r for r in recs if any(k.startswith("val/") for k in r)]
    if not evals:
        return None
    last = evals[-1]
    speeds = [r["perf/tokens_per_s"] for r in recs if "perf/tokens_per_s" in r]
    speeds = speeds[len(speeds) // 10:]
    cfg = yaml.safe_load((run_dir / "config.yaml").read_text())
    params: dict = {}
    for r in recs:
        params.update({k[len("params/"):]: v for k, v in r.items() if k.startswith("params/")})
    return {"run_name": run_dir.name, "step": last["step"], "steps": cfg["steps"],
            "val": {k[len("val/"):]: v for k, v in last.items() if k.startswith("val/")},
            "tokens_per_s": float(np.median(speeds)) if speeds else None, "params": params}


def report(sweep_dir: Path) -> str:
    results = load_results(sweep_dir)
    if not results:
        return "(no finished runs)"
    sets = sorted({k.split("/")[0] for r in results for k in r["val"] if k.endswith("/bpb")})
    head = ["| run | seeds | " + " | ".join(f"{s} bpb" for s in sets) + " | mean bpb | steps | tok/s |",
            "|---|---|" + "---|" * len(sets) + "---|---|---|"]
    rows = []
    for name, runs in group_seeds(results).items():
        bpb = {s: float(np.mean([r["val"][f"{s}/bpb"] for r in runs if f"{s}/bpb" in r["val"]] or [np.nan]))
               for s in sets}
        mean = float(np.mean(list(bpb.values()))) if bpb else float("nan")
        speed = np.mean([r["tokens_per_s"] if r["tokens_per_s"] is not None else np.nan for r in runs])
        cells = " | ".join(f"{bpb[s]:.4f}" for s in sets)
        rows.append((mean, f"| {name} | {len(runs)} | {cells} | {mean:.4f} | {runs[0]['steps']} | {speed / 1e3:.0f}K |"))
    return "\n".join(head + [r for _, r in sorted(rows, key=lambda t: (np.isnan(t[0]), t[0]))])


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep")
    ap.add_argument("--report", action="store_true", help="only print the summary table")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--output-dir", default="runs/sweeps")
    args = ap.parse_args(argv)
    sweep = yaml.safe_load(Path(args.sweep).read_text())
    sweep_dir = Path(args.output_dir) / sweep["name"]
    if not args.report:
        for run in plan(sweep):
            run_all([run], sweep_dir, "myk_llm_b200.train", dry_run=args.dry_run)
            s = None if args.dry_run else summarize(sweep_dir / run[0])
            if s is not None and s["step"] >= s["steps"]:
                (sweep_dir / run[0] / "results.json").write_text(json.dumps(s, indent=1))
    print(report(sweep_dir))


if __name__ == "__main__":
    main()
