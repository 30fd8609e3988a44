"""Endless packed batches of fresh arithmetic problems.  Each problem is its own
document (document-masked attention); the loss covers the completion and EOS only;
the tail of a row is padding in a separate unsupervised document."""

from __future__ import annotations

import random
from typing import Iterator

import torch
from torch.utils.data import DataLoader, IterableDataset, get_worker_info

from ..data.config import IGNORE_INDEX, Batch
from .tasks import CharTokenizer, TaskConfig, add_fillers, render, sample_problem


def encode_example(tokenizer: CharTokenizer, prompt: str, completion: str) -> tuple[list[int], list[int]]:
    """Token ids and next-token targets, supervised only where the next token belongs
    to the completion."""
    ids = tokenizer.encode(prompt + completion)
    targets = [IGNORE_INDEX] * len(ids)
    targets[len(prompt) - 1:len(ids) - 1] = ids[len(prompt):]
    return ids, targets


class PackedArithmetic(IterableDataset):
    def __init__(self, task: TaskConfig, batch_rows: int, row_len: int, seed: int) -> None:
        super().__init__()
        self.task, self.batch_rows, self.row_len, self.seed = task, batch_rows, row_len, seed
        self.tokenizer = CharTokenizer()

    def _example(self, rng: random.Random) -> tuple[list[int], list[int]]:
        prompt, comp = render(*sample_problem(rng, self.task), self.task)
        prompt = add_fillers(prompt, rng, self.task.filler_prob, self.task.max_fillers)
        ex = encode_example(self.tokenizer, prompt, comp)
        if len(ex[0]) > self.row_len:
            raise ValueError(f"an example of {len(ex[0])} tokens exceeds row_len {self.row_len}")
        return ex

    def rows(self, rng: random.Random) -> Iterator[tuple[list[int], list[int], list[int]]]:
        carry = None
        while True:
            ids, tg, lens = [], [], []
            while True:
                ex = carry if carry is not None else self._example(rng)
                carry = None
                if len(ids) + len(ex[0]) > self.row_len:
                    carry = ex
                    break
                ids += ex[0]
                tg += ex[1]
                lens.append(len(ex[0]))
            pad = self.row_len - len(ids)
            if pad:
                ids += [self.tokenizer.pad_id] * pad
                tg += [IGNORE_INDEX] * pad
                lens.append(pad)
            yield ids, tg, lens

    def __iter__(self) -> Iterator[Batch]:
        w = get_worker_info()
        rows = self.rows(random.Random(self.seed * 1000 + (w.id if w else 0)))
        while True:
            chunk = [next(rows) for _ in range(self.batch_rows)]
            yield Batch(torch.tensor([r[0] for r in chunk], dtype=torch.long),
                        torch.tensor([r[1] for r in chunk], dtype=torch.long),
                        [torch.tensor(r[2], dtype=torch.int32) for r in chunk])


def build_loader(task: TaskConfig, batch_rows: int, row_len: int, seed: int, num_workers: int) -> DataLoader:
    return DataLoader(PackedArithmetic(task, batch_rows, row_len, seed), batch_size=None, num_workers=num_workers,
                      pin_memory=torch.cuda.is_available(), persistent_workers=num_workers > 0,
                      prefetch_factor=8 if num_workers > 0 else None)
