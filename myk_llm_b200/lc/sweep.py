"""Retrieval sweeps: the grid runner of :mod:`myk_llm_b200.utils.sweep` plus tables of
effective context length.

    python -m myk_llm_b200.lc.sweep configs/lc/sweeps/length.yaml
    python -m myk_llm_b200.lc.sweep configs/lc/sweeps/length.yaml --report --at 8192

``eff@90`` / ``eff@50``: the longest length up to which every evaluated length stays at
>= 90% / 50% accuracy.  ``--at L`` adds accuracy by needle depth and by hop count at L and
the final scans (hop extrapolation, core iteration counts).
"""

from __future__ import annotations

import argparse
from pathlib import Path

import numpy as np
import yaml

from ..utils.sweep import SEED_SUFFIX, load_results, plan, run_all

METRICS = ("accuracy", "accuracy_late")


def effective_length(acc: dict[str, float], threshold: float) -> int:
    best = 0
    for L in sorted(acc, key=int):
        if acc[L] < threshold:
            break
        best = int(L)
    return best


def _k(n: float) -> str:
    return f"{n / 1024:.3g}K" if n >= 1024 else f"{n:.0f}"


def _groups(results: list[dict]) -> dict[str, dict[str, list[dict]]]:
    g: dict[str, dict[str, list[dict]]] = {}
    for r in results:
        g.setdefault(r["run_name"].split("-")[0], {}).setdefault(SEED_SUFFIX.sub("", r["run_name"]), []).append(r)
    return g


def report(sweep_dir: Path, metric: str = "accuracy", at: int | None = None) -> str:
    results = [r for r in load_results(sweep_dir) if r.get(metric)]
    if not results:
        return f"(no finished runs with {metric})"
    lines = []
    for task, configs in _groups(results).items():
        lengths = sorted({int(k) for runs in configs.values() for r in runs for k in r[metric]})
        train_len = next(iter(configs.values()))[0]["train_len"]
        lines += [f"\n### {task}, {metric} (trained on <= {train_len} tokens)\n",
                  "| run | seeds | eff@90 | eff@50 | " + " | ".join(_k(n) for n in lengths) + " | min |",
                  "|---|---|---|---|" + "---|" * len(lengths) + "---|"]
        rows = []
        for name, runs in configs.items():
            e90 = np.mean([effective_length(r[metric], 0.9) for r in runs])
            e50 = np.mean([effective_length(r[metric], 0.5) for r in runs])
            cells = " | ".join(f"{100 * np.mean([r[metric].get(str(n), np.nan) for r in runs]):.0f}" for n in lengths)
            mins = np.mean([r["train_minutes"] for r in runs])
            rows.append(((-e50, -e90, name), f"| {name} | {len(runs)} | {_k(e90)} | {_k(e50)} | {cells} | {mins:.1f} |"))
        lines += [r for _, r in sorted(rows)]
        if at is not None:
            lines += detail(configs, at) + scan_table(configs, at)
    return "\n".join(lines)


def detail(configs: dict[str, list[dict]], length: int) -> list[str]:
    key = str(length)
    at = {n: [r for r in rs if key in r.get("depth", {})] for n, rs in configs.items()}
    at = {n: rs for n, rs in at.items() if rs}
    if not at:
        return [f"\n(no evaluation at length {length})"]
    nb = len(next(iter(at.values()))[0]["depth"][key])
    lines = [f"\nAccuracy by needle depth at {_k(length)} (0 = start of the context)\n",
             "| run | " + " | ".join(f"{100 * i // nb}%" for i in range(nb)) + " |", "|---|" + "---|" * nb]
    for n, rs in sorted(at.items()):
        d = np.nanmean([r["depth"][key] for r in rs], axis=0)
        lines.append(f"| {n} | " + " | ".join(f"{100 * x:.0f}" for x in d) + " |")
    hops = sorted({h for rs in at.values() for r in rs for h in r["hops"][key]}, key=int)
    if len(hops) > 1:
        lines += [f"\nAccuracy by hop count at {_k(length)}\n", "| run | " + " | ".join(f"{h} hops" for h in hops) + " |",
                  "|---|" + "---|" * len(hops)]
        for n, rs in sorted(at.items()):
            lines.append(f"| {n} | " + " | ".join(
                f"{100 * np.mean([r['hops'][key].get(h, np.nan) for r in rs]):.0f}" for h in hops) + " |")
    return lines


def scan_table(configs: dict[str, list[dict]], length: int) -> list[str]:
    key = str(length)
    cells: dict[tuple[str, int | None], list[dict]] = {}
    for n, rs in configs.items():
        for r in rs:
            for sc in r.get("scan", []):
                if key in sc["hops"]:
                    cells.setdefault((n, sc["iterations"]), []).append(sc["hops"][key])
    if not cells:
        return []
    hops = sorted({h for rs in cells.values() for r in rs for h in r}, key=int)
    lines = [f"\nFinal scan at {_k(length)}: accuracy by hop count per core iteration count\n",
             "| run | iterations | seeds | " + " | ".join(f"{h} hops" for h in hops) + " |",
             "|---|---|---|" + "---|" * len(hops)]
    for (n, it), rs in sorted(cells.items(), key=lambda kv: (kv[0][0], kv[0][1] or 0)):
        lines.append(f"| {n} | {it or '-'} | {len(rs)} | " + " | ".join(
            f"{100 * np.mean([r.get(h, np.nan) for r in rs]):.0f}" for h in hops) + " |")
    return lines


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("sweep")
    ap.add_argument("--report", action="store_true")
    ap.add_argument("--metric", choices=METRICS, default=None)
    ap.add_argument("--at", type=int, default=None)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--output-dir", default="runs/lc")
    args = ap.parse_args(argv)
    sweep = yaml.safe_load(Path(args.sweep).read_text(encoding="utf-8"))
    sweep_dir = Path(args.output_dir) / sweep["name"]
    if not args.report:
        run_all(plan(sweep), sweep_dir, "myk_llm_b200.lc.train", args.dry_run)
    metrics = [args.metric] if args.metric else list(METRICS)
    tables = [report(sweep_dir, m, args.at if m == metrics[0] else None) for m in metrics]
    table = "\n".join(t for t in tables if not t.startswith("(no finished")) or "(no finished runs)"
    print(table)
    if sweep_dir.exists():
        (sweep_dir / "summary.md").write_text(table + "\n", encoding="utf-8")


if __name__ == "__main__":
    main()
