"""Endless packed batches of fresh retrieval (and copy) examples: rows of ``task.max_len``
tokens, one document per example, the loss on the answers only (packing:
:mod:`myk_llm_b200.utils.testbed`)."""

from __future__ import annotations

from typing import Iterator

import numpy as np
from torch.utils.data import DataLoader

from ..data.config import IGNORE_INDEX
from ..utils.testbed import PackedExamples, packed_loader
from .tasks import PAD, Example, TaskConfig, make_copy_example, make_example


def answer_targets(example: Example) -> np.ndarray:
    """Next-token targets set only at the positions that predict an answer token."""
    targets = np.full(len(example.ids), IGNORE_INDEX, dtype=np.int64)
    for start, end in example.answers:
        targets[start - 1:end - 1] = example.ids[start:end]
    return targets


def retrieval_examples(task: TaskConfig, rng: np.random.Generator) -> Iterator[tuple[np.ndarray, np.ndarray]]:
    while True:
        if task.copy_fraction and rng.random() < task.copy_fraction:
            ex = make_copy_example(rng, task)
        else:
            ex = make_example(rng, task, task.sample_length(rng), task.sample_records(rng))
        yield ex.ids, answer_targets(ex)


class PackedRetrieval(PackedExamples):
    def __init__(self, task: TaskConfig, batch_rows: int, seed: int) -> None:
        super().__init__(lambda rng: retrieval_examples(task, rng), batch_rows, task.max_len, PAD, seed)
        self.task = task


def build_loader(task: TaskConfig, batch_rows: int, seed: int, num_workers: int) -> DataLoader:
    return packed_loader(PackedRetrieval(task, batch_rows, seed), num_workers)
