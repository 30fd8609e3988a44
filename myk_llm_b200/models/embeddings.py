"""Input embeddings: token table plus optional hashed n-gram tables.

The n-gram hash must map token windows to the same bucket rows as the upstream model,
otherwise a checkpoint's n-gram tables would be read at the wrong rows.  The rolling
hash (reference: ``src/myk_llm/model/embeddings.py:14-30``) is therefore reproduced
exactly: start from the order n, and for offsets 0..n-1 (the token at the position, then
the ones before it) do ``h = h * M[offset % 4] + token + 1; h ^= h >> 29`` in wrapping
int64, then ``h mod num_buckets``.  Missing left context uses the id ``vocab_size``.
Table k's row b is row ``k * num_buckets + b`` of the stacked tables.

On CUDA the hash, the gather of every order and the sum run in one kernel
(:func:`myk_llm_b200.ops.ngram_lookup`).
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn

from .. import ops
from .config import ModelConfig, NgramEmbeddingConfig

HASH_MULTIPLIERS = (0x1F3D5B79A2C4E681, 0x0DDC0FFEEBADF00D, 0x1B873593CC9E2D51, 0x0000000100000001B3)


def ngram_bucket_ids(tokens: torch.Tensor, order: int, context: int, num_buckets: int) -> torch.Tensor:
    """Bucket ids (batch, seq) of the ``order`` tokens ending at each position of
    ``tokens[:, context:]`` (the first ``context`` columns are left context)."""
    seq = tokens.size(1) - context
    h = torch.full_like(tokens[:, context:], order)
    for off in range(order):
        tok = tokens[:, context - off : context - off + seq]
        h = h * HASH_MULTIPLIERS[off % len(HASH_MULTIPLIERS)] + tok + 1
        h = h ^ (h >> 29)
    return torch.remainder(h, num_buckets)


class NgramEmbedding(nn.Module):
    def __init__(self, config: NgramEmbeddingConfig, vocab_size: int, hidden_size: int) -> None:
        super().__init__()
        self.orders = list(config.orders)
        self.num_buckets = config.num_buckets
        self.sentinel = vocab_size
        self.tables = nn.ModuleList(nn.Embedding(config.num_buckets, config.dim) for _ in self.orders)
        self.layers = list(config.layers)
        project = config.dim != hidden_size or self.layers != [0]
        self.projs = nn.ModuleList(
            nn.Linear(config.dim, hidden_size, bias=False) if project else nn.Identity() for _ in self.layers)
        # Lazy (sparse-update) training replaces the table lookup with its own rows.
        self.row_source: Callable[[torch.Tensor], torch.Tensor] | None = None

    @property
    def context(self) -> int:
        return max(self.orders) - 1

    def forward(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None) -> dict[int, torch.Tensor]:
        feats = self.lookup(input_ids, prefix_ids)
        out = {}
        for layer, proj in zip(self.layers, self.projs):
            out[layer] = ops.linear(feats, proj.weight) if isinstance(proj, nn.Linear) else feats
        return out

    def _with_context(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None) -> torch.Tensor:
        bsz, ctx = input_ids.size(0), self.context
        left = torch.full((bsz, ctx), self.sentinel, dtype=input_ids.dtype, device=input_ids.device)
        if prefix_ids is not None and prefix_ids.size(1) > 0:
            tail = prefix_ids[:, -ctx:]
            left[:, ctx - tail.size(1):] = tail
        return torch.cat([left, input_ids], dim=1)

    def row_ids(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None = None) -> torch.Tensor:
        """(orders, batch, seq) ids into the stacked tables."""
        tokens = self._with_context(input_ids, prefix_ids)
        return torch.stack([
            ngram_bucket_ids(tokens, n, self.context, self.num_buckets) + k * self.num_buckets
            for k, n in enumerate(self.orders)])

    def lookup(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None) -> torch.Tensor:
        if self.row_source is not None:
            return self.row_source(self.row_ids(input_ids, prefix_ids))
        if input_ids.is_cuda:
            tokens = self._with_context(input_ids, prefix_ids)
            return ops.ngram_lookup(tokens, [t.weight for t in self.tables], self.orders, self.context,
                                    self.num_buckets)
        ids = self.row_ids(input_ids, prefix_ids)
        return sum(t(ids[k] - k * self.num_buckets) for k, t in enumerate(self.tables))


class Embeddings(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.token = nn.Embedding(config.vocab_size, config.hidden_size)
        self.ngram = NgramEmbedding(config.ngram, config.vocab_size, config.hidden_size) if config.ngram.orders else None

    @property
    def context(self) -> int:
        return self.ngram.context if self.ngram is not None else 0

    def forward(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None = None):
        updates = self.ngram(input_ids, prefix_ids) if self.ngram is not None else {}
        return ops.embedding(input_ids, self.token.weight), updates
