"""Grids of pretraining runs (``python -m myk_llm_b200.train``) and their summary table.

A sweep file (the format of :mod:`myk_llm_b200.utils.sweep`, shared with the reference's
``scripts/sweep_train.py``) expands into one run per combination of its axes; a run whose
directory already holds ``results.json`` is skipped, so re-running the command resumes.
When a run reaches its last step its summary is written to ``<sweep>/<run>/results.json``:
final validation metrics, median throughput after the first tenth of the log, and the
parameter counts.  The report merges seeds (runs named ``...-s<k>``) and sorts by mean
bits per byte::

    python -m myk_llm_b200.train.sweep_train configs/ngram-small/sweeps/main.yaml
    python -m myk_llm_b200.train.sweep_train configs/ngram-small/sweeps/main.yaml --report
"""

from __future__ import annotations

import argparse
import json
import statistics
from dataclasses import asdict, dataclass, field
from pathlib import Path

import yaml

from ..utils.sweep import group_seeds, load_results, plan, run_all


@dataclass
class RunSummary:
    run_name: str
    step: int
    steps: int
    val: dict[str, float] = field(default_factory=dict)
    tokens_per_s: float | None = None
    params: dict[str, float] = field(default_factory=dict)

    @property
    def finished(self) -> bool:
        return self.step >= self.steps


def summarize(run_dir: Path) -> dict | None:
    """The summary of a run from one pass over its metrics log (None before its first
    validation)."""
    log = Path(run_dir) / "metrics.jsonl"
    if not log.exists():
        return None
    last_eval: dict | None = None
    speeds: list[float] = []
    params: dict[str, float] = {}
    with log.open(encoding="utf-8") as fh:
        for line in fh:
            if not line.strip():
                continue
            rec = json.loads(line)
            if any(k.startswith("val/") for k in rec):
                last_eval = rec
            if "perf/tokens_per_s" in rec:
                speeds.append(rec["perf/tokens_per_s"])
            for k, v in rec.items():
                if k.startswith("params/"):
                    params[k[len("params/"):]] = v
    if last_eval is None:
        return None
    steady = speeds[len(speeds) // 10:]
    steps = yaml.safe_load((Path(run_dir) / "config.yaml").read_text())["steps"]
    return asdict(RunSummary(
        run_name=Path(run_dir).name, step=last_eval["step"], steps=steps,
        val={k[len("val/"):]: v for k, v in last_eval.items() if k.startswith("val/")},
        tokens_per_s=float(statistics.median(steady)) if steady else None, params=params))


def _mean(xs: list[float]) -> float:
    xs = [x for x in xs if x is not None]
    return sum(xs) / len(xs) if xs else float("nan")


def report(sweep_dir: Path) -> str:
    """Markdown table: one row per configuration (seeds merged), best mean bpb first."""
    results = load_results(sweep_dir)
    if not results:
        return "(no finished runs)"
    sets = sorted({k.rsplit("/", 1)[0] for r in results for k in r["val"] if k.endswith("/bpb")})
    header = ["run", "seeds", *[f"{s} bpb" for s in sets], "mean bpb", "steps", "tok/s"]
    rows = []
    for name, runs in group_seeds(results).items():
        per_set = [_mean([r["val"].get(f"{s}/bpb") for r in runs]) for s in sets]
        mean = _mean(per_set) if per_set else float("nan")
        speed = _mean([r["tokens_per_s"] for r in runs])
        cells = [name, str(len(runs)), *[f"{x:.4f}" for x in per_set], f"{mean:.4f}", str(runs[0]["steps"]),
                 f"{speed / 1e3:.0f}K"]
        rows.append((mean != mean, mean, cells))  # NaN means last
    rows.sort(key=lambda r: (r[0], r[1]))
    lines = ["| " + " | ".join(header) + " |", "|" + "---|" * len(header)]
    lines += ["| " + " | ".join(cells) + " |" for _, _, cells in rows]
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep")
    ap.add_argument("--report", action="store_true", help="only print the summary table")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--output-dir", default="runs/sweeps")
    args = ap.parse_args(argv)
    spec = yaml.safe_load(Path(args.sweep).read_text())
    sweep_dir = Path(args.output_dir) / spec["name"]
    if not args.report:
        for run in plan(spec):
            run_all([run], sweep_dir, "myk_llm_b200.train", dry_run=args.dry_run)
            if args.dry_run:
                continue
            summary = summarize(sweep_dir / run[0])
            if summary is not None and summary["step"] >= summary["steps"]:
                (sweep_dir / run[0] / "results.json").write_text(json.dumps(summary, indent=1))
    print(report(sweep_dir))


if __name__ == "__main__":
    main()
