"""Endless packed batches of fresh arithmetic problems: every problem is its own document
(document-masked attention), the loss covers the completion and the end marker only, and
row tails are unsupervised padding documents (packing: :mod:`myk_llm_b200.utils.testbed`)."""

from __future__ import annotations

import random
from typing import Iterator

import numpy as np
from torch.utils.data import DataLoader

from ..data.config import IGNORE_INDEX
from ..utils.testbed import PackedExamples, packed_loader
from .tasks import CharTokenizer, TaskConfig, add_fillers, render, sample_problem


def encode_example(tokenizer: CharTokenizer, prompt: str, completion: str) -> tuple[list[int], list[int]]:
    """Ids of ``prompt + completion`` and next-token targets that are set only where the
    next token is part of the completion."""
    ids = tokenizer.encode(prompt + completion)
    first = len(prompt) - 1  # the position that predicts the completion's first character
    return ids, [IGNORE_INDEX] * first + ids[first + 1:] + [IGNORE_INDEX]


def arithmetic_examples(task: TaskConfig, rng: np.random.Generator) -> Iterator[tuple[np.ndarray, np.ndarray]]:
    """Endless (ids, targets) examples; the problem stream is a ``random.Random`` seeded
    from ``rng`` so problems match Python's integer sampling exactly."""
    tok = CharTokenizer()
    draw = random.Random(int(rng.integers(0, 2 ** 63)))
    while True:
        prompt, completion = render(*sample_problem(draw, task), task)
        prompt = add_fillers(prompt, draw, task.filler_prob, task.max_fillers)
        ids, targets = encode_example(tok, prompt, completion)
        yield np.asarray(ids, dtype=np.int64), np.asarray(targets, dtype=np.int64)


class PackedArithmetic(PackedExamples):
    def __init__(self, task: TaskConfig, batch_rows: int, row_len: int, seed: int) -> None:
        super().__init__(lambda rng: arithmetic_examples(task, rng), batch_rows, row_len, CharTokenizer().pad_id,
                         seed)
        self.task = task


def build_loader(task: TaskConfig, batch_rows: int, row_len: int, seed: int, num_workers: int) -> DataLoader:
    return packed_loader(PackedArithmetic(task, batch_rows, row_len, seed), num_workers)
