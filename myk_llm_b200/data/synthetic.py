"""Synthetic packed-document data (the benchmark configurations' data source).

Each row of ``seq_len + 1`` tokens packs documents whose lengths are drawn from a
geometric distribution with mean ``mean_doc_len`` (capped at the row length), token ids
uniform over the vocabulary except the EOS id, and an EOS after every document.  As
with real shards, a document end inside the window is a cut point: the EOS target that
crosses the seam is masked and ``seqlens`` gives the per-row document lengths.

The stream is a deterministic function of (seed, global step), and every rank slices the
same global batch, so the state to checkpoint is the step counter and resuming on a
different number of GPUs continues the same global sequence.
"""

from __future__ import annotations

from typing import Any, Iterator

import numpy as np
import torch

from .config import IGNORE_INDEX, Batch, DataConfig, collate


def packed_row(rng: np.random.Generator, seq_len: int, vocab: int, mean: int, eos: int,
               document_masking: bool = True) -> dict[str, np.ndarray]:
    n = seq_len + 1
    toks = rng.integers(0, vocab - 1, size=n, dtype=np.int64)
    toks[toks >= eos] += 1  # skip the EOS id
    ends = []
    pos = 0
    p = 1.0 / max(1, mean)
    while pos < n:
        length = int(min(rng.geometric(p), n))
        pos += length
        if pos <= n:
            toks[pos - 1] = eos
            ends.append(pos)
    row = {"input_ids": toks[:-1], "targets": toks[1:].copy()}
    if document_masking:
        cuts = np.asarray([e for e in ends if 0 < e < seq_len], dtype=np.int64)
        # the EOS closing a document at position e-1 has its target (the next document's
        # first token) masked: it crosses the seam
        if len(cuts):
            row["targets"][cuts - 1] = IGNORE_INDEX
        row["seqlens"] = np.diff(np.concatenate(([0], cuts, [seq_len]))).astype(np.int32)
    return row


class SyntheticLoader:
    """Rank-sliced, resumable batches of packed random documents."""

    def __init__(self, config: DataConfig, rank: int = 0, world_size: int = 1) -> None:
        self.config, self.rank, self.world_size = config, rank, world_size
        self.step = 0

    def _row(self, global_row: int) -> dict[str, np.ndarray]:
        c, s = self.config, self.config.synthetic
        rng = np.random.default_rng([c.seed, global_row])
        return packed_row(rng, c.seq_len, s.vocab_size, s.mean_doc_len, s.eos_id, c.document_masking)

    def rows_of(self, step: int) -> list[int]:
        """Global row indices of this rank's micro-batch at ``step``: a fixed slice of the
        global batch, or, with ``synthetic.balance_ranks``, the rows that a longest-first
        assignment gives this rank so that every rank's attention work (sum over its rows of
        the squared document lengths) is about equal.  Every rank computes the same
        assignment from the same global batch."""
        c = self.config
        micro, world = c.micro_batch_size, self.world_size
        first = step * world * micro
        if not c.synthetic.balance_ranks or world == 1 or not c.document_masking:
            return [first + self.rank * micro + i for i in range(micro)]
        cost = []
        for g in range(first, first + world * micro):
            lens = self._row(g)["seqlens"].astype(np.float64)
            cost.append(float((lens * lens).sum()))
        order = sorted(range(world * micro), key=lambda i: (-cost[i], i))
        load, count = [0.0] * world, [0] * world
        mine = []
        for i in order:
            r = min((r for r in range(world) if count[r] < micro), key=lambda r: (load[r], r))
            load[r] += cost[i]
            count[r] += 1
            if r == self.rank:
                mine.append(first + i)
        return sorted(mine)

    def batch_at(self, step: int) -> Batch:
        return collate([self._row(g) for g in self.rows_of(step)])

    def next_batch(self) -> Batch:
        b = self.batch_at(self.step)
        self.step += 1
        return b

    def __iter__(self) -> Iterator[Batch]:
        while True:
            yield self.next_batch()

    def state_dict(self) -> dict[str, Any]:
        return {"kind": "synthetic", "step": self.step}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.step = int(state["step"])

    def close(self) -> None:
        pass
