"""Loss parity of a low-precision training run against bf16: the same model, data and
seed trained twice for N steps through ``Trainer.train_step``, once with
``parallel.float8`` set and once without, and the two loss curves compared (one GPU).

    python -m myk_llm_b200.train.loss_parity configs/baseline/1b_mxfp8.yaml --steps 200
    python -m myk_llm_b200.train.loss_parity configs/baseline/1b_mxfp8.yaml --steps 200 --json out.json

The reference checks one training step of fp8 / MXFP8 against bf16
(``tests/test_float8.py:59-86``) and reports longer bf16-vs-fp8 runs in its notes
(``notes/fp8.md:75-81``); this runner produces the longer comparison for any config.
Data: the config's data source (the benchmark configs use synthetic packed documents);
both runs see identical batches.  Reported: the per-step losses, the mean absolute and
relative gap over the last quarter of the steps, and each run's throughput.
"""

from __future__ import annotations

import argparse
import json
import time

import torch

from ..configuration import load_config
from ..parallel.distributed import DistInfo
from .config import TrainConfig
from .trainer import Trainer


def run(config: TrainConfig, steps: int, float8: str) -> dict:
    """``steps`` optimizer steps with ``parallel.float8 = float8``; per-step losses."""
    from dataclasses import replace

    cfg = replace(config, steps=steps, parallel=replace(config.parallel, float8=float8))
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    trainer = Trainer(cfg, DistInfo(0, 1, 0, dev))
    loader = iter(trainer.loader)
    losses = []
    torch.cuda.synchronize() if dev.type == "cuda" else None
    start = time.perf_counter()
    for step in range(1, steps + 1):
        batches = [next(loader) for _ in range(trainer.grad_accum)]
        out = trainer.train_step(batches, step)
        losses.append(out["loss"].detach())
    if dev.type == "cuda":
        torch.cuda.synchronize()
    seconds = time.perf_counter() - start
    loader_close = getattr(trainer.loader, "close", None)
    if loader_close is not None:
        loader_close()
    values = [float(x) for x in losses]
    return {"float8": float8, "losses": values, "tokens_per_s": steps * trainer.tokens_per_step / seconds}


def compare(a: list[float], b: list[float]) -> dict:
    tail = max(1, len(a) // 4)
    da = [abs(x - y) for x, y in zip(a[-tail:], b[-tail:])]
    return {"last_quarter_mean_abs_gap": sum(da) / tail,
            "last_quarter_mean_rel_gap": sum(d / max(1e-9, abs(y)) for d, y in zip(da, b[-tail:])) / tail,
            "final": {"test": a[-1], "bf16": b[-1]}}


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config")
    ap.add_argument("overrides", nargs="*")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--float8", default=None, help="recipe of the test run (default: the config's)")
    ap.add_argument("--json", default="", help="write the full result here")
    args = ap.parse_args(argv)
    cfg = load_config(TrainConfig, args.config, args.overrides)
    recipe = args.float8 or cfg.parallel.float8
    if recipe == "none":
        raise SystemExit("the config trains in bf16; pass --float8 <recipe>")
    test = run(cfg, args.steps, recipe)
    base = run(cfg, args.steps, "none")
    result = {"config": args.config, "steps": args.steps, "test": test, "bf16": base,
              "gap": compare(test["losses"], base["losses"])}
    every = max(1, args.steps // 10)
    print(f"| step | {recipe} loss | bf16 loss |\n|---|---|---|")
    for i in list(range(every - 1, args.steps, every)):
        print(f"| {i + 1} | {test['losses'][i]:.4f} | {base['losses'][i]:.4f} |")
    g = result["gap"]
    print(f"\nlast quarter: mean |gap| {g['last_quarter_mean_abs_gap']:.4f} "
          f"({100 * g['last_quarter_mean_rel_gap']:.2f}%); throughput {recipe} {test['tokens_per_s']:,.0f} tok/s, "
          f"bf16 {base['tokens_per_s']:,.0f} tok/s")
    if args.json:
        with open(args.json, "w") as fh:
            json.dump(result, fh, indent=1)


if __name__ == "__main__":
    main()
