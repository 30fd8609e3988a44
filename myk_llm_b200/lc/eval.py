"""Exact-match retrieval accuracy on a grid of context length x needle depth (x hops).

Scoring is teacher-forced: a query is correct when the argmax at every answer position
equals the target, which is exactly greedy-decoding exact match, but takes one forward
pass per batch.  Only the answer positions go through the LM head.
"""

from __future__ import annotations

import contextlib
from dataclasses import replace

import numpy as np
import torch

from ..models import MykLLM
from .tasks import Example, TaskConfig, make_example


def _amp(device):
    return torch.autocast("cuda", dtype=torch.bfloat16) if device.type == "cuda" else contextlib.nullcontext()


def answer_positions(examples: list[Example], device) -> tuple[torch.Tensor, torch.Tensor, list[tuple[int, int]]]:
    rows, pos, spans = [], [], []
    for r, ex in enumerate(examples):
        for s, e in ex.answers:
            spans.append((len(pos), len(pos) + e - s))
            rows += [r] * (e - s)
            pos += range(s - 1, e - 1)
    return torch.tensor(rows, device=device), torch.tensor(pos, device=device), spans


def score_batch(model: MykLLM, examples: list[Example], iterations: int | None = None) -> list[bool]:
    """Per-query exact match for equal-length examples (one document per row)."""
    dev = model.device
    ids = torch.from_numpy(np.stack([e.ids for e in examples])).to(dev)
    rows, pos, spans = answer_positions(examples, dev)
    kw = {} if iterations is None else {"iterations": iterations}
    with _amp(dev):
        hidden = model(ids, seqlens=[torch.tensor([ids.size(1)])] * ids.size(0), **kw).hidden
        pred = model.logits(hidden[rows, pos]).argmax(-1)
    hit = (pred == ids[rows, pos + 1]).cpu().tolist()
    return [all(hit[a:b]) for a, b in spans]


@torch.no_grad()
def evaluate(model: MykLLM, task: TaskConfig, lengths: list[int], queries: int, seed: int,
             tokens_per_batch: int = 65536, iterations: int | None = None, hops: list[int] | None = None) -> dict:
    """{"accuracy": {L: acc}, "depth": {L: [acc per depth bucket]}, "hops": {L: {h: acc}}}."""
    was = model.training
    model.eval()
    if hops is not None:
        task = replace(task, hops=hops)
    out: dict[str, dict] = {"accuracy": {}, "depth": {}, "hops": {}}
    nb = task.depth_buckets
    for L in lengths:
        rng = np.random.default_rng([seed, L])
        exs = [make_example(rng, task, L) for _ in range(-(-queries // task.num_queries))]
        per = max(1, tokens_per_batch // L)
        ok: list[bool] = []
        for s in range(0, len(exs), per):
            ok += score_batch(model, exs[s:s + per], iterations)
        depths = [d for e in exs for d in e.depths]
        hs = [h for e in exs for h in e.hops]
        hits, counts = np.zeros(nb), np.zeros(nb)
        for good, d in zip(ok, depths):
            b = min(int(d * nb), nb - 1)
            hits[b] += good
            counts[b] += 1
        out["accuracy"][L] = float(np.mean(ok))
        out["depth"][L] = [float(h / c) if c else float("nan") for h, c in zip(hits, counts)]
        out["hops"][L] = {h: float(np.mean([g for g, k in zip(ok, hs) if k == h])) for h in sorted(set(hs))}
    model.train(was)
    return out
