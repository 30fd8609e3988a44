"""Train a character-level model on arithmetic (one GPU).

    python -m myk_llm_b200.arith.train configs/arith/add.yaml [key.path=value ...]

Writes ``<output_dir>/<run_name>/``: config.yaml, metrics.jsonl, model.pt and results.json
(final exact-match accuracy per operand length, the in-distribution mean, and the mean of
the evaluations in the second half of training, a steadier summary at long lengths).
The YAML schema (``ArithConfig``) and the results keys are the reference's
(``src/myk_llm/arith/train.py``) so sweep files and reports carry over.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass, field
from pathlib import Path

import torch

from ..configuration import dump_yaml, load_config
from ..models import ModelConfig
from ..train.config import ObjectiveConfig, OptimizerConfig, ScheduleConfig
from ..train.metrics import MetricsLogger
from ..train.objectives import Objective
from ..train.optim import build_optimizers
from ..utils.testbed import LoopSettings, TestbedLoop
from .data import build_loader
from .model import ArithModel, DigitEmbeddingConfig, evaluate_lengths
from .tasks import TaskConfig


@dataclass
class ArithConfig:
    run_name: str = "arith"
    output_dir: str = "runs/arith"
    seed: int = 0
    task: TaskConfig = field(default_factory=TaskConfig)
    model: ModelConfig = field(default_factory=ModelConfig)
    digit_embedding: DigitEmbeddingConfig = field(default_factory=DigitEmbeddingConfig)
    steps: int = 5000
    batch_rows: int = 64
    row_len: int = 1024
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    schedule: ScheduleConfig = field(default_factory=ScheduleConfig)
    objective: ObjectiveConfig = field(default_factory=ObjectiveConfig)
    compile: bool = True  # accepted for config compatibility; the kernels need no compiler
    num_workers: int = 4
    log_interval: int = 100
    eval_interval: int = 1000
    eval_examples: int = 200
    final_eval_examples: int = 1000


class _Evaluations:
    """Periodic accuracy (plain prompts, and prompts with fillers when the task uses them)
    and the second-half record used for ``accuracy_late``."""

    def __init__(self, config: ArithConfig, model: ArithModel, metrics: MetricsLogger) -> None:
        self.config, self.model, self.metrics = config, model, metrics
        self.lengths = config.task.eval_lengths()
        self.variants = {"": False, "fillers_": True} if config.task.filler_prob > 0 else {"": False}
        self.late: dict[str, list[dict[int, float]]] = {k: [] for k in self.variants}

    def __call__(self, step: int) -> None:
        for prefix, fillers in self.variants.items():
            acc = evaluate_lengths(self.model, self.config.task, self.lengths, self.config.eval_examples, seed=step,
                                   fillers=fillers)
            self.metrics.log(step, {f"{prefix}acc/{d}": a for d, a in acc.items()})
            if step >= self.config.steps // 2:
                self.late[prefix].append(acc)

    def final(self) -> dict[str, dict[int, float]]:
        return {prefix: evaluate_lengths(self.model, self.config.task, self.lengths, self.config.final_eval_examples,
                                         seed=12345, fillers=fillers)
                for prefix, fillers in self.variants.items()}


def train(config: ArithConfig, device: str | None = None) -> dict:
    torch.manual_seed(config.seed)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    if config.digit_embedding.enabled and config.task.filler_prob > 0:
        raise ValueError("the digit embedding counts runs of consecutive digits, which fillers split")
    run_dir = Path(config.output_dir) / config.run_name
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "config.yaml").write_text(dump_yaml(config), encoding="utf-8")
    model = ArithModel(config.model, config.digit_embedding).to(dev)
    optimizers = build_optimizers(model.lm, config.optimizer)
    if model.digit_embed is not None:  # the digit table trains with AdamW, no decay
        optimizers[-1].add_param_group({"params": [model.digit_embed.weight], "weight_decay": 0.0,
                                        "lr": config.optimizer.lr})
    metrics = MetricsLogger(run_dir / "metrics.jsonl")
    params = model.lm.num_parameters(exclude_embeddings=True)
    print(f"[{config.run_name}] {params / 1e6:.2f}M non-embedding params, {config.batch_rows}x{config.row_len} "
          f"tokens/step, {config.steps} steps", flush=True)
    loop = TestbedLoop(LoopSettings(config.steps, config.log_interval, config.eval_interval,
                                    config.optimizer.grad_clip, config.run_name),
                       model, optimizers, config.schedule, Objective(config.objective, dev),
                       lambda batch, head: model(batch, head), metrics, dev)
    evals = _Evaluations(config, model, metrics)
    loop.run(iter(build_loader(config.task, config.batch_rows, config.row_len, config.seed, config.num_workers)),
             evals)
    torch.save({"config": dump_yaml(config), "state_dict": model.state_dict()}, run_dir / "model.pt")
    finals = evals.final()
    acc = finals[""]
    inside = [a for d, a in acc.items() if d <= config.task.train_digits]
    results = {"run_name": config.run_name, "accuracy": acc, "train_digits": config.task.train_digits,
               "in_distribution": sum(inside) / max(1, len(inside)), "non_embedding_params": params,
               "train_minutes": loop.minutes}
    for prefix, scores in finals.items():
        if prefix:
            results[f"{prefix}accuracy"] = scores
        history = evals.late[prefix]
        if history:
            results[f"{prefix}accuracy_late"] = {d: sum(h[d] for h in history) / len(history) for d in evals.lengths}
        metrics.log(config.steps, {f"final_{prefix}acc/{d}": a for d, a in scores.items()})
    metrics.close()
    (run_dir / "results.json").write_text(json.dumps(results, indent=2), encoding="utf-8")
    return results


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config", nargs="?", default=None)
    ap.add_argument("overrides", nargs="*")
    args = ap.parse_args(argv)
    train(load_config(ArithConfig, args.config, args.overrides))


if __name__ == "__main__":
    main()
