"""Grid sweeps for the research testbeds (arith, lc).

A sweep file names one base config per task and axes of named override lists; every
combination is one run in a fresh process.  Runs that already wrote ``results.json``
are skipped, so an interrupted sweep resumes by running the same command again::

    name: format-position
    configs: {add: configs/arith/add.yaml, mul: configs/arith/mul.yaml}
    axes:
      format: {direct: [task.format=direct], cot: [task.format=cot]}
    overrides: [steps=3000]

(the sweep file format of the reference's ``src/myk_llm/arith/sweep.py:10-16``).
"""

from __future__ import annotations

import itertools
import json
import re
import subprocess
import sys
from pathlib import Path

SEED_SUFFIX = re.compile(r"-s\d+$")


def plan(sweep: dict) -> list[tuple[str, str, list[str]]]:
    """[(run name, base config, overrides)] for every task x axis combination."""
    axes = sweep.get("axes", {}) or {}
    runs = []
    for task, cfg in sweep["configs"].items():
        for combo in itertools.product(*[list(v.items()) for v in axes.values()]):
            name = "-".join([task] + [label for label, _ in combo])
            ov = list(sweep.get("overrides", []) or []) + [o for _, group in combo for o in group]
            runs.append((name, cfg, ov))
    return runs


def run_all(runs, sweep_dir: Path, module: str, dry_run: bool = False) -> list[str]:
    """Run each plan entry as ``python -m module`` (log in <run>/train.log); returns the
    names of runs that failed."""
    failed = []
    for i, (name, cfg, ov) in enumerate(runs, 1):
        if (sweep_dir / name / "results.json").exists():
            print(f"[{i}/{len(runs)}] {name}: done, skipping", flush=True)
            continue
        cmd = [sys.executable, "-m", module, cfg, *ov, f"run_name={name}", f"output_dir={sweep_dir}"]
        print(f"[{i}/{len(runs)}] {name}: {' '.join(ov)}", flush=True)
        if dry_run:
            continue
        log = sweep_dir / name / "train.log"
        log.parent.mkdir(parents=True, exist_ok=True)
        with log.open("w") as fh:
            code = subprocess.call(cmd, stdout=fh, stderr=subprocess.STDOUT)
        if code:
            failed.append(name)
            print(f"  failed (exit {code}); see {log}", flush=True)
    return failed


def load_results(sweep_dir: Path) -> list[dict]:
    return [json.loads(p.read_text()) for p in sorted(Path(sweep_dir).glob("*/results.json"))]


def group_seeds(results: list[dict], key: str = "run_name") -> dict[str, list[dict]]:
    """Runs whose names differ only by a trailing ``-s<k>`` are seeds of one config."""
    out: dict[str, list[dict]] = {}
    for r in results:
        out.setdefault(SEED_SUFFIX.sub("", r[key]), []).append(r)
    return out
