"""Exact-match retrieval accuracy on a grid of context length x needle depth (x hops).

Scoring is teacher-forced: a query counts as correct when the argmax at every position
that predicts one of its answer tokens equals that token, which is exactly greedy
exact match but needs one forward pass per batch; only those positions go through the LM
head.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

from ..models import MykLLM
from ..utils.testbed import autocast_for
from .tasks import Example, TaskConfig, make_example


def answer_positions(examples: list[Example], device) -> tuple[torch.Tensor, torch.Tensor, list[tuple[int, int]]]:
    """(row, position) of every answer-predicting position, and each query's [lo, hi) slice
    of those lists."""
    rows, cols, spans = [], [], []
    for r, ex in enumerate(examples):
        for start, end in ex.answers:
            spans.append((len(cols), len(cols) + end - start))
            cols.extend(range(start - 1, end - 1))
            rows.extend([r] * (end - start))
    return torch.tensor(rows, device=device), torch.tensor(cols, device=device), spans


def score_batch(model: MykLLM, examples: list[Example], iterations: int | None = None) -> list[bool]:
    """Exact match per query for examples of one length (one document per row)."""
    dev = model.device
    ids = torch.as_tensor(np.stack([e.ids for e in examples]), device=dev)
    rows, cols, spans = answer_positions(examples, dev)
    extra = {"iterations": iterations} if iterations is not None else {}
    with autocast_for(dev):
        hidden = model(ids, seqlens=[torch.tensor([ids.shape[1]])] * ids.shape[0], **extra).hidden
        hit = model.logits(hidden[rows, cols]).argmax(-1) == ids[rows, cols + 1]
    hit = hit.cpu().numpy()
    return [bool(hit[lo:hi].all()) for lo, hi in spans]


def _by_depth(correct: list[bool], depths: list[float], buckets: int) -> list[float]:
    idx = np.minimum((np.asarray(depths) * buckets).astype(int), buckets - 1)
    hits = np.bincount(idx, weights=np.asarray(correct, dtype=float), minlength=buckets)
    counts = np.bincount(idx, minlength=buckets)
    return [float(h / c) if c else float("nan") for h, c in zip(hits, counts)]


@torch.no_grad()
def evaluate(model: MykLLM, task: TaskConfig, lengths: list[int], queries: int, seed: int,
             tokens_per_batch: int = 65536, iterations: int | None = None, hops: list[int] | None = None) -> dict:
    """{"accuracy": {L: acc}, "depth": {L: [acc per depth bucket]}, "hops": {L: {h: acc}}}."""
    training = model.training
    model.eval()
    if hops is not None:
        task = replace(task, hops=hops)
    result: dict[str, dict] = {"accuracy": {}, "depth": {}, "hops": {}}
    for length in lengths:
        rng = np.random.default_rng([seed, length])
        examples = [make_example(rng, task, length) for _ in range(-(-queries // task.num_queries))]
        per_batch = max(1, tokens_per_batch // length)
        correct = [ok for lo in range(0, len(examples), per_batch)
                   for ok in score_batch(model, examples[lo:lo + per_batch], iterations)]
        depths = [d for e in examples for d in e.depths]
        hop_of = [h for e in examples for h in e.hops]
        result["accuracy"][length] = float(np.mean(correct))
        result["depth"][length] = _by_depth(correct, depths, task.depth_buckets)
        result["hops"][length] = {h: float(np.mean([c for c, k in zip(correct, hop_of) if k == h]))
                                  for h in sorted(set(hop_of))}
    model.train(training)
    return result
