"""Retrieval sweeps: the grid runner of :mod:`myk_llm_b200.utils.sweep` and tables of
effective context length.

    python -m myk_llm_b200.lc.sweep configs/lc/sweeps/length.yaml
    python -m myk_llm_b200.lc.sweep configs/lc/sweeps/length.yaml --report --at 8192

``eff@90`` / ``eff@50``: the longest length up to which every evaluated length stays at
>= 90% / 50% accuracy.  ``--at L`` adds accuracy by needle depth and by hop count at L and
the final scans (hop extrapolation, core iteration counts).  The report layout follows the
reference's ``src/myk_llm/lc/sweep.py``.
"""

from __future__ import annotations

import argparse
from collections import defaultdict
from pathlib import Path

import numpy as np
import yaml

from ..utils.sweep import SEED_SUFFIX, load_results, plan, run_all

METRICS = ("accuracy", "accuracy_late")


def effective_length(acc: dict[str, float], threshold: float) -> int:
    """The longest length L such that every evaluated length <= L scores >= threshold."""
    ordered = sorted(acc.items(), key=lambda kv: int(kv[0]))
    passing = 0
    for length, value in ordered:
        if value < threshold:
            return passing
        passing = int(length)
    return passing


def _tok(n: float) -> str:
    return f"{n / 1024:.3g}K" if n >= 1024 else f"{n:.0f}"


def _md(header: list[str], rows: list[list[str]]) -> list[str]:
    return ["| " + " | ".join(header) + " |", "|" + "---|" * len(header)] + ["| " + " | ".join(r) + " |" for r in rows]


def _by_task(results: list[dict]) -> dict[str, dict[str, list[dict]]]:
    """task (name prefix) -> configuration (name without seed suffix) -> runs."""
    tree: dict[str, dict[str, list[dict]]] = defaultdict(lambda: defaultdict(list))
    for r in results:
        tree[r["run_name"].split("-")[0]][SEED_SUFFIX.sub("", r["run_name"])].append(r)
    return tree


def _mean(xs) -> float:
    xs = [x for x in xs if x is not None]
    return float(np.mean(xs)) if xs else float("nan")


def report(sweep_dir: Path, metric: str = "accuracy", at: int | None = None) -> str:
    results = [r for r in load_results(sweep_dir) if r.get(metric)]
    if not results:
        return f"(no finished runs with {metric})"
    out: list[str] = []
    for task, configs in _by_task(results).items():
        every = [r for runs in configs.values() for r in runs]
        lengths = sorted({int(k) for r in every for k in r[metric]})
        out.append(f"\n### {task}, {metric} (trained on <= {every[0]['train_len']} tokens)\n")
        ranked = []
        for name, runs in configs.items():
            e90 = _mean(effective_length(r[metric], 0.9) for r in runs)
            e50 = _mean(effective_length(r[metric], 0.5) for r in runs)
            cells = [f"{100 * _mean(r[metric].get(str(n)) for r in runs):.0f}" for n in lengths]
            row = [name, str(len(runs)), _tok(e90), _tok(e50), *cells, f"{_mean(r['train_minutes'] for r in runs):.1f}"]
            ranked.append(((-e50, -e90, name), row))
        out += _md(["run", "seeds", "eff@90", "eff@50", *map(_tok, lengths), "min"], [r for _, r in sorted(ranked)])
        if at is not None:
            out += detail(configs, at) + scan_table(configs, at)
    return "\n".join(out)


def detail(configs: dict[str, list[dict]], length: int) -> list[str]:
    """Accuracy by needle depth (and by hop count when several) at ``length``."""
    key = str(length)
    runs_at = {n: [r for r in rs if key in r.get("depth", {})] for n, rs in configs.items()}
    runs_at = {n: rs for n, rs in sorted(runs_at.items()) if rs}
    if not runs_at:
        return [f"\n(no evaluation at length {length})"]
    buckets = len(next(iter(runs_at.values()))[0]["depth"][key])
    out = [f"\nAccuracy by needle depth at {_tok(length)} (0 = start of the context)\n"]
    out += _md(["run", *[f"{100 * i // buckets}%" for i in range(buckets)]],
               [[n] + [f"{100 * v:.0f}" for v in np.nanmean([r["depth"][key] for r in rs], axis=0)]
                for n, rs in runs_at.items()])
    hop_keys = sorted({h for rs in runs_at.values() for r in rs for h in r["hops"][key]}, key=int)
    if len(hop_keys) > 1:
        out.append(f"\nAccuracy by hop count at {_tok(length)}\n")
        out += _md(["run", *[f"{h} hops" for h in hop_keys]],
                   [[n] + [f"{100 * _mean(r['hops'][key].get(h) for r in rs):.0f}" for h in hop_keys]
                    for n, rs in runs_at.items()])
    return out


def scan_table(configs: dict[str, list[dict]], length: int) -> list[str]:
    """The final scans at ``length``: accuracy by hop count per core iteration count."""
    key = str(length)
    cells: dict[tuple[str, int | None], list[dict]] = defaultdict(list)
    for name, runs in configs.items():
        for r in runs:
            for scan in r.get("scan", []):
                if key in scan["hops"]:
                    cells[(name, scan["iterations"])].append(scan["hops"][key])
    if not cells:
        return []
    hop_keys = sorted({h for seeds in cells.values() for s in seeds for h in s}, key=int)
    rows = [[name, str(it or "-"), str(len(seeds)), *[f"{100 * _mean(s.get(h) for s in seeds):.0f}" for h in hop_keys]]
            for (name, it), seeds in sorted(cells.items(), key=lambda kv: (kv[0][0], kv[0][1] or 0))]
    return [f"\nFinal scan at {_tok(length)}: accuracy by hop count per core iteration count\n"] + \
        _md(["run", "iterations", "seeds", *[f"{h} hops" for h in hop_keys]], rows)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep")
    ap.add_argument("--report", action="store_true")
    ap.add_argument("--metric", choices=METRICS, default=None)
    ap.add_argument("--at", type=int, default=None)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--output-dir", default="runs/lc")
    args = ap.parse_args(argv)
    spec = yaml.safe_load(Path(args.sweep).read_text(encoding="utf-8"))
    sweep_dir = Path(args.output_dir) / spec["name"]
    if not args.report:
        run_all(plan(spec), sweep_dir, "myk_llm_b200.lc.train", args.dry_run)
    metrics = [args.metric] if args.metric else list(METRICS)
    tables = [report(sweep_dir, m, args.at if i == 0 else None) for i, m in enumerate(metrics)]
    text = "\n".join(t for t in tables if not t.startswith("(no finished")) or "(no finished runs)"
    print(text)
    if sweep_dir.exists():
        (sweep_dir / "summary.md").write_text(text + "\n", encoding="utf-8")


if __name__ == "__main__":
    main()
