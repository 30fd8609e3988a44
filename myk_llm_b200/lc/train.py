"""Train a small model on synthetic long-context retrieval (one GPU).

    python -m myk_llm_b200.lc.train configs/lc/needle.yaml [key.path=value ...]

Writes ``<output_dir>/<run_name>/``: config.yaml, metrics.jsonl, model.pt and results.json
(exact-match accuracy per context length, per needle depth and per hop count; the step at
which retrieval was learned; optional final scans over hop counts and, for looped models,
core iteration counts).  ``LcConfig`` and the results keys are the reference's
(``src/myk_llm/lc/train.py``) so sweeps and reports carry over.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from ..configuration import dump_yaml, load_config
from ..models import ModelConfig, MykLLM
from ..train.config import ObjectiveConfig, OptimizerConfig, ScheduleConfig
from ..train.metrics import MetricsLogger
from ..train.objectives import Objective
from ..train.optim import build_optimizers
from ..utils.testbed import LoopSettings, TestbedLoop
from .data import build_loader
from .eval import evaluate
from .tasks import VOCAB_SIZE, TaskConfig

LEARNED_AT = 0.9  # in-distribution accuracy at which retrieval counts as learned


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
    compile: bool = True            # accepted for config compatibility; the kernels need no compiler
    num_workers: int = 4
    log_interval: int = 100
    eval_interval: int = 1000
    eval_queries: int = 200
    final_eval_queries: int = 1000
    eval_iterations: int = 0        # looped models: core iterations of every evaluation (0: default)
    scan_iterations: list[int] = field(default_factory=list)
    scan_lengths: list[int] = field(default_factory=list)


def late_mean(late: list[tuple[int, dict[int, float]]], learned: int | None, lengths: list[int]) -> dict:
    """Mean accuracy per length over the second-half evaluations from the learned step on."""
    kept = [acc for step, acc in late if learned is None or step >= learned]
    return {L: float(np.mean([a[L] for a in kept])) for L in lengths} if kept else {}


def _check(config: LcConfig) -> None:
    if config.model.vocab_size < VOCAB_SIZE:
        raise ValueError(f"model.vocab_size must be at least {VOCAB_SIZE}")
    if max(config.task.eval_lengths + [config.task.max_len]) > config.model.max_seq_len:
        raise ValueError("model.max_seq_len must cover the longest evaluation length")
    if (config.eval_iterations or config.scan_iterations) and not config.model.loop.core:
        raise ValueError("eval_iterations / scan_iterations need a looped model")


class _Progress:
    """Periodic evaluations: the learned step and the second-half accuracies."""

    def __init__(self, config: LcConfig, model: MykLLM, metrics: MetricsLogger) -> None:
        self.config, self.model, self.metrics = config, model, metrics
        self.lengths = list(config.task.eval_lengths)
        self.iterations = config.eval_iterations or None
        self.learned: int | None = None
        self.late: list[tuple[int, dict[int, float]]] = []

    def in_distribution(self, acc: dict[int, float]) -> float:
        inside = [a for L, a in acc.items() if L <= self.config.task.max_len]
        return float(np.mean(inside)) if inside else float("nan")

    def __call__(self, step: int) -> None:
        res = evaluate(self.model, self.config.task, self.lengths, self.config.eval_queries, seed=step,
                       iterations=self.iterations)
        self.metrics.log(step, {f"acc/{L}": a for L, a in res["accuracy"].items()})
        if self.learned is None and self.in_distribution(res["accuracy"]) >= LEARNED_AT:
            self.learned = step
        if step >= self.config.steps // 2:
            self.late.append((step, res["accuracy"]))


def train(config: LcConfig, device: str | None = None) -> dict:
    torch.manual_seed(config.seed)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    _check(config)
    task = config.task
    run_dir = Path(config.output_dir) / config.run_name
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "config.yaml").write_text(dump_yaml(config), encoding="utf-8")
    model = MykLLM(config.model).to(dev)
    if config.init_from:
        model.load_state_dict(torch.load(config.init_from, map_location=dev)["state_dict"])
    metrics = MetricsLogger(run_dir / "metrics.jsonl")
    params = model.num_parameters(exclude_embeddings=True)
    print(f"[{config.run_name}] {params / 1e6:.2f}M non-embedding params, {config.batch_rows}x{task.max_len} "
          f"tokens/step, {config.steps} steps", flush=True)
    loop = TestbedLoop(LoopSettings(config.steps, config.log_interval, config.eval_interval,
                                    config.optimizer.grad_clip, config.run_name),
                       model, build_optimizers(model, config.optimizer), config.schedule,
                       Objective(config.objective, dev),
                       lambda batch, head: model(batch.input_ids, seqlens=batch.seqlens, head=head), metrics, dev)
    progress = _Progress(config, model, metrics)
    if config.steps:
        loop.run(iter(build_loader(task, config.batch_rows, config.seed, config.num_workers)), progress)
    torch.save({"config": dump_yaml(config), "state_dict": model.state_dict()}, run_dir / "model.pt")
    final = evaluate(model, task, progress.lengths, config.final_eval_queries, seed=12345,
                     iterations=progress.iterations)
    metrics.log(config.steps, {f"final_acc/{L}": a for L, a in final["accuracy"].items()})
    scans = []
    if task.eval_hops or config.scan_iterations:
        for iters in config.scan_iterations or [None]:
            sc = evaluate(model, task, config.scan_lengths or progress.lengths, config.final_eval_queries,
                          seed=12345, iterations=iters, hops=task.eval_hops or None)
            scans.append({"iterations": iters, "accuracy": sc["accuracy"], "hops": sc["hops"]})
    metrics.close()
    learned = progress.learned
    if learned is None and progress.in_distribution(final["accuracy"]) >= LEARNED_AT:
        learned = config.steps
    results = {"run_name": config.run_name, "train_len": task.max_len, **final,
               "accuracy_late": late_mean(progress.late, learned, progress.lengths),
               "in_distribution": progress.in_distribution(final["accuracy"]), "learned_step": learned,
               "scan": scans, "non_embedding_params": params, "train_minutes": loop.minutes}
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
