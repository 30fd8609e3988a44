"""Train a character-level model on arithmetic (one GPU).

    python -m myk_llm_b200.arith.train configs/arith/add.yaml [key.path=value ...]

Writes ``<output_dir>/<run_name>/``: config.yaml, metrics.jsonl, model.pt and
results.json (final exact-match accuracy per operand length; also the mean over the
evaluations of the second half of training, a steadier summary for long lengths).
"""

from __future__ import annotations

import argparse
import contextlib
import json
import time
from dataclasses import dataclass, field
from pathlib import Path

import torch

from .. import ops
from ..configuration import dump_yaml, load_config
from ..models import ModelConfig
from ..train.config import ObjectiveConfig, OptimizerConfig, ScheduleConfig
from ..train.metrics import MetricsLogger
from ..train.objectives import Objective
from ..train.optim import build_optimizers, lr_multiplier, set_lr
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
    compile: bool = True
    num_workers: int = 4
    log_interval: int = 100
    eval_interval: int = 1000
    eval_examples: int = 200
    final_eval_examples: int = 1000


def train(config: ArithConfig, device: str | None = None) -> dict:
    torch.manual_seed(config.seed)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    run_dir = Path(config.output_dir) / config.run_name
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "config.yaml").write_text(dump_yaml(config), encoding="utf-8")
    if config.digit_embedding.enabled and config.task.filler_prob > 0:
        raise ValueError("the digit embedding counts runs of consecutive digits, which fillers split")
    model = ArithModel(config.model, config.digit_embedding).to(dev)
    opts = build_optimizers(model.lm, config.optimizer)
    if model.digit_embed is not None:
        opts[-1].add_param_group({"params": [model.digit_embed.weight], "weight_decay": 0.0,
                                  "lr": config.optimizer.lr})
    base = [[g["lr"] for g in o.param_groups] for o in opts]
    objective = Objective(config.objective, dev)
    loader = iter(build_loader(config.task, config.batch_rows, config.row_len, config.seed, config.num_workers))
    metrics = MetricsLogger(run_dir / "metrics.jsonl")
    lengths = config.task.eval_lengths()
    variants = {"": False, "fillers_": True} if config.task.filler_prob > 0 else {"": False}
    late: dict[str, list[dict[int, float]]] = {k: [] for k in variants}
    params = model.lm.num_parameters(exclude_embeddings=True)
    print(f"[{config.run_name}] {params / 1e6:.2f}M non-embedding params, {config.batch_rows}x{config.row_len} "
          f"tokens/step, {config.steps} steps", flush=True)
    amp = torch.autocast("cuda", dtype=torch.bfloat16) if dev.type == "cuda" else contextlib.nullcontext()
    t_start = t_win = time.perf_counter()
    loss_sum = tok_sum = 0.0
    for step in range(1, config.steps + 1):
        set_lr(opts, base, lr_multiplier(step, config.steps, config.schedule))
        batch = next(loader).to(dev)
        n = batch.num_targets
        with amp:
            out = model(batch, objective.head(batch, float(n)))
        out.loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), config.optimizer.grad_clip or float("inf"))
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
        ops.invalidate_weight_cache()
        loss_sum += float(out.sums["ce"])
        tok_sum += n
        if step % config.log_interval == 0:
            dt = time.perf_counter() - t_win
            rec = {"train/loss": loss_sum / max(1, tok_sum),
                   "perf/tokens_per_s": config.log_interval * batch.input_ids.numel() / dt}
            metrics.log(step, rec)
            print(f"[{config.run_name}] step {step} loss {rec['train/loss']:.4f} "
                  f"{rec['perf/tokens_per_s']:,.0f} tok/s", flush=True)
            loss_sum = tok_sum = 0.0
            t_win = time.perf_counter()
        if config.eval_interval and step % config.eval_interval == 0 and step != config.steps:
            for prefix, fill in variants.items():
                acc = evaluate_lengths(model, config.task, lengths, config.eval_examples, seed=step, fillers=fill)
                metrics.log(step, {f"{prefix}acc/{d}": a for d, a in acc.items()})
                if step >= config.steps // 2:
                    late[prefix].append(acc)
            t_win = time.perf_counter()
    torch.save({"config": dump_yaml(config), "state_dict": model.state_dict()}, run_dir / "model.pt")
    finals = {p: evaluate_lengths(model, config.task, lengths, config.final_eval_examples, seed=12345, fillers=f)
              for p, f in variants.items()}
    acc = finals[""]
    in_d = [a for d, a in acc.items() if d <= config.task.train_digits]
    results = {"run_name": config.run_name, "accuracy": acc, "train_digits": config.task.train_digits,
               "in_distribution": sum(in_d) / max(1, len(in_d)), "non_embedding_params": params,
               "train_minutes": (time.perf_counter() - t_start) / 60}
    for p, fin in finals.items():
        if p:
            results[f"{p}accuracy"] = fin
        if late[p]:
            results[f"{p}accuracy_late"] = {d: sum(a[d] for a in late[p]) / len(late[p]) for d in lengths}
        metrics.log(config.steps, {f"final_{p}acc/{d}": a for d, a in fin.items()})
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
