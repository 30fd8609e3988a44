"""Endless packed batches of fresh retrieval (and copy) examples: rows of task.max_len
tokens, one document per example, loss on the answers only."""

from __future__ import annotations

from typing import Iterator

import numpy as np
import torch
from torch.utils.data import DataLoader, IterableDataset, get_worker_info

from ..data.config import IGNORE_INDEX, Batch
from .tasks import PAD, Example, TaskConfig, make_copy_example, make_example


def answer_targets(example: Example) -> np.ndarray:
    tg = np.full(len(example.ids), IGNORE_INDEX, dtype=np.int64)
    for s, e in example.answers:
        tg[s - 1:e - 1] = example.ids[s:e]
    return tg


class PackedRetrieval(IterableDataset):
    def __init__(self, task: TaskConfig, batch_rows: int, seed: int) -> None:
        super().__init__()
        self.task, self.batch_rows, self.seed = task, batch_rows, seed

    def _example(self, rng: np.random.Generator) -> Example:
        t = self.task
        if t.copy_fraction and rng.random() < t.copy_fraction:
            return make_copy_example(rng, t)
        return make_example(rng, t, t.sample_length(rng), t.sample_records(rng))

    def rows(self, rng: np.random.Generator) -> Iterator[tuple[np.ndarray, np.ndarray, list[int]]]:
        width, carry = self.task.max_len, None
        while True:
            ids, tg, lens, used = [], [], [], 0
            while True:
                ex = carry if carry is not None else self._example(rng)
                carry = None
                if used + len(ex.ids) > width:
                    carry = ex
                    break
                ids.append(ex.ids)
                tg.append(answer_targets(ex))
                lens.append(len(ex.ids))
                used += len(ex.ids)
            if used < width:
                ids.append(np.full(width - used, PAD, dtype=np.int64))
                tg.append(np.full(width - used, IGNORE_INDEX, dtype=np.int64))
                lens.append(width - used)
            yield np.concatenate(ids), np.concatenate(tg), lens

    def __iter__(self) -> Iterator[Batch]:
        w = get_worker_info()
        rows = self.rows(np.random.default_rng([self.seed, w.id if w else 0]))
        while True:
            chunk = [next(rows) for _ in range(self.batch_rows)]
            yield Batch(torch.from_numpy(np.stack([c[0] for c in chunk])),
                        torch.from_numpy(np.stack([c[1] for c in chunk])),
                        [torch.tensor(c[2], dtype=torch.int32) for c in chunk])


def build_loader(task: TaskConfig, batch_rows: int, seed: int, num_workers: int) -> DataLoader:
    return DataLoader(PackedRetrieval(task, batch_rows, seed), batch_size=None, num_workers=num_workers,
                      pin_memory=torch.cuda.is_available(), persistent_workers=num_workers > 0,
                      prefetch_factor=8 if num_workers > 0 else None)
