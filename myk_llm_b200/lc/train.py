"""Train a small model on synthetic long-context retrieval (one GPU).

    python -m myk_llm_b200.lc.train configs/lc/needle.yaml [key.path=value ...]

Writes ``<output_dir>/<run_name>/``: config.yaml, metrics.jsonl, model.pt and results.json
(exact-match accuracy per context length, per needle depth and per hop count; the step
at which retrieval was learned; optional final scans over hop counts and, for looped
models, core iteration counts).
"""

from __future__ import annotations

import argparse
import contextlib
import json
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from .. import ops
from ..configuration import dump_yaml, load_config
from ..models import MykLLM, ModelConfig
from ..train.config import ObjectiveConfig, OptimizerConfig, ScheduleConfig
from ..train.metrics import MetricsLogger
from ..train.objectives import Objective
from ..train.optim import build_optimizers, lr_multiplier, set_lr
from .data import build_loader
from .eval import evaluate
from .tasks import VOCAB_SIZE, TaskConfig


@dataclass
class LcConfig:
    run_name: str = "lc"
    output_dir: str = "runs/lc"
    seed: int = 0
    task: TaskConfig = field(default_factory=TaskConfig)
    model: ModelConfig = field(default_factory=ModelConfig)
    init_from: str = ""             # model.pt of an earlier run (curriculum); steps=0: evaluate only
    steps: int = 5000
    batch_rows: int = 32            # rows of task.max_len tokens per step
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    schedule: ScheduleConfig = field(default_factory=ScheduleConfig)
    objective: ObjectiveConfig = field(default_factory=ObjectiveConfig)
    compile: bool = True
    num_workers: int = 4
    log_interval: int = 100
    eval_interval: int = 1000
    eval_queries: int = 200
    final_eval_queries: int = 1000
    eval_iterations: int = 0        # looped models: core iterations of every evaluation (0: default)
    scan_iterations: list[int] = field(default_factory=list)
    scan_lengths: list[int] = field(default_factory=list)


def late_mean(late: list[tuple[int, dict[int, float]]], learned: int | None, lengths: list[int]) -> dict:
    """Mean accuracy per length over the second-half evaluations from the transition on."""
    kept = [a for s, a in late if learned is None or s >= learned]
    return {L: float(np.mean([a[L] for a in kept])) for L in lengths} if kept else {}


def train(config: LcConfig, device: str | None = None) -> dict:
    torch.manual_seed(config.seed)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    task = config.task
    if config.model.vocab_size < VOCAB_SIZE:
        raise ValueError(f"model.vocab_size must be at least {VOCAB_SIZE}")
    if max(task.eval_lengths + [task.max_len]) > config.model.max_seq_len:
        raise ValueError("model.max_seq_len must cover the longest evaluation length")
    if (config.eval_iterations or config.scan_iterations) and not config.model.loop.core:
        raise ValueError("eval_iterations / scan_iterations need a looped model")
    run_dir = Path(config.output_dir) / config.run_name
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "config.yaml").write_text(dump_yaml(config), encoding="utf-8")
    model = MykLLM(config.model).to(dev)
    if config.init_from:
        model.load_state_dict(torch.load(config.init_from, map_location=dev)["state_dict"])
    opts = build_optimizers(model, config.optimizer)
    base = [[g["lr"] for g in o.param_groups] for o in opts]
    objective = Objective(config.objective, dev)
    loader = iter(build_loader(task, config.batch_rows, config.seed, config.num_workers))
    metrics = MetricsLogger(run_dir / "metrics.jsonl")
    lengths = list(task.eval_lengths)
    iters = config.eval_iterations or None
    late: list[tuple[int, dict[int, float]]] = []
    learned = None

    def in_dist(acc: dict[int, float]) -> float:
        v = [a for L, a in acc.items() if L <= task.max_len]
        return float(np.mean(v)) if v else float("nan")

    params = model.num_parameters(exclude_embeddings=True)
    print(f"[{config.run_name}] {params / 1e6:.2f}M non-embedding params, {config.batch_rows}x{task.max_len} "
          f"tokens/step, {config.steps} steps", flush=True)
    amp = torch.autocast("cuda", dtype=torch.bfloat16) if dev.type == "cuda" else contextlib.nullcontext()
    t0 = tw = time.perf_counter()
    loss_sum = tok_sum = 0.0
    for step in range(1, config.steps + 1):
        set_lr(opts, base, lr_multiplier(step, config.steps, config.schedule))
        batch = next(loader).to(dev)
        n = batch.num_targets
        with amp:
            out = model(batch.input_ids, seqlens=batch.seqlens, head=objective.head(batch, float(max(1, n))))
        out.loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), config.optimizer.grad_clip or float("inf"))
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
        ops.invalidate_weight_cache()
        loss_sum += float(out.sums["ce"])
        tok_sum += n
        if step % config.log_interval == 0:
            rec = {"train/loss": loss_sum / max(1, tok_sum),
                   "perf/tokens_per_s": config.log_interval * batch.input_ids.numel() / (time.perf_counter() - tw)}
            metrics.log(step, rec)
            print(f"[{config.run_name}] step {step} loss {rec['train/loss']:.4f}", flush=True)
            loss_sum = tok_sum = 0.0
            tw = time.perf_counter()
        if config.eval_interval and step % config.eval_interval == 0 and step != config.steps:
            res = evaluate(model, task, lengths, config.eval_queries, seed=step, iterations=iters)
            metrics.log(step, {f"acc/{L}": a for L, a in res["accuracy"].items()})
            if learned is None and in_dist(res["accuracy"]) >= 0.9:
                learned = step
            if step >= config.steps // 2:
                late.append((step, res["accuracy"]))
            tw = time.perf_counter()
    torch.save({"config": dump_yaml(config), "state_dict": model.state_dict()}, run_dir / "model.pt")
    final = evaluate(model, task, lengths, config.final_eval_queries, seed=12345, iterations=iters)
    metrics.log(config.steps, {f"final_acc/{L}": a for L, a in final["accuracy"].items()})
    scans = []
    if task.eval_hops or config.scan_iterations:
        for it in config.scan_iterations or [None]:
            sc = evaluate(model, task, config.scan_lengths or lengths, config.final_eval_queries, seed=12345,
                          iterations=it, hops=task.eval_hops or None)
            scans.append({"iterations": it, "accuracy": sc["accuracy"], "hops": sc["hops"]})
    metrics.close()
    if learned is None and in_dist(final["accuracy"]) >= 0.9:
        learned = config.steps
    results = {"run_name": config.run_name, "train_len": task.max_len, **final,
               "accuracy_late": late_mean(late, learned, lengths), "in_distribution": in_dist(final["accuracy"]),
               "learned_step": learned, "scan": scans, "non_embedding_params": params,
               "train_minutes": (time.perf_counter() - t0) / 60}
    (run_dir / "results.json").write_text(json.dumps(results, indent=2), encoding="utf-8")
    return results


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config", nargs="?", default=None)
    ap.add_argument("overrides", nargs="*")
    args = ap.parse_args(argv)
    train(load_config(LcConfig, args.config, args.overrides))


if __name__ == "__main__":
    main()
