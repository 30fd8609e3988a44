"""Input embeddings: the token table plus optional hashed n-gram tables.

The n-gram bucket function is part of the checkpoint contract (a checkpoint's table rows
must be read for the same token windows in both frameworks), so it is the reference's
(``src/myk_llm/model/embeddings.py:14-30``): start from the order ``n`` and, for offsets
``0 .. n-1`` (the token at the position, then the ones before it), ``h = h * M[o % 4] +
token + 1; h ^= h >> 29`` in wrapping int64, then ``h mod num_buckets``; left context
missing at the start of a sequence reads as the id ``vocab_size``.  Order ``k``'s table
row ``b`` is row ``k * num_buckets + b`` of the stacked tables.

On CUDA one kernel per direction does the whole n-gram embedding
(``ngram_embed_fwd`` hashes every order, gathers the rows and sums them;
``ngram_embed_bwd`` scatter-adds the gradient into every order's rows); the statements
below are the CPU path and the test oracle.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn

from .. import ops
from .config import ModelConfig, NgramEmbeddingConfig

HASH_MULTIPLIERS = (0x1F3D5B79A2C4E681, 0x0DDC0FFEEBADF00D, 0x1B873593CC9E2D51, 0x0000000100000001B3)


def ngram_bucket_ids(tokens: torch.Tensor, order: int, context: int, num_buckets: int) -> torch.Tensor:
    """Buckets (batch, seq) of the ``order``-token windows ending at each position of
    ``tokens[:, context:]`` (the first ``context`` columns are left context)."""
    seq = tokens.shape[1] - context
    windows = [tokens[:, context - o:context - o + seq] for o in range(order)]
    h = torch.full_like(windows[0], order)
    for o, tok in enumerate(windows):
        h = h * HASH_MULTIPLIERS[o % 4] + tok + 1
        h ^= h >> 29
    return h.remainder(num_buckets)


class _NgramEmbed(torch.autograd.Function):
    """Fused hash + gather + sum on the GPU; the backward adds into each table's
    ``main_grad`` (or a fresh gradient)."""

    @staticmethod
    def forward(ctx, tokens, context: int, orders: tuple[int, ...], *tables):
        shards = getattr(tables[0], "_mykb_table", None)  # row-sharded over the ranks (parallel/sharded.py)
        if shards is not None:
            out, rows = shards.forward(tokens.contiguous(), context)
        else:
            out, rows = ops.ext().ngram_embed_fwd(tokens.contiguous(), list(tables), list(orders), context)
        ctx.save_for_backward(rows)
        ctx.tables = tables
        ctx.shards = shards
        ctx.lead = tokens.shape[0], tokens.shape[1] - context
        return out.view(*ctx.lead, out.shape[-1])

    @staticmethod
    def backward(ctx, dout):
        (rows,) = ctx.saved_tensors
        if ctx.shards is not None:  # added into the owners' gradient rows
            ctx.shards.backward(rows, dout.reshape(-1, dout.shape[-1]).float().contiguous())
            return (None, None, None, *(None for _ in ctx.tables))
        grads, fresh = [], []
        for t in ctx.tables:
            main = getattr(t, "main_grad", None)
            g = main if main is not None else torch.zeros(t.shape, dtype=torch.float32, device=t.device)
            grads.append(g)
            fresh.append(None if main is not None else g)
        ops.ext().ngram_embed_bwd(rows, dout.reshape(-1, dout.shape[-1]).float().contiguous(), grads)
        return (None, None, None, *fresh)


class NgramEmbedding(nn.Module):
    """One table per n-gram order (summed), fed into the blocks listed in ``layers``,
    each through its own projection (identity when the table width is the model width
    and only block 0 receives it)."""

    def __init__(self, config: NgramEmbeddingConfig, vocab_size: int, hidden_size: int) -> None:
        super().__init__()
        self.orders = list(config.orders)
        self.num_buckets = config.num_buckets
        self.sentinel = vocab_size
        self.layers = list(config.layers)
        self.tables = nn.ModuleList([nn.Embedding(config.num_buckets, config.dim) for _ in self.orders])
        identity = config.dim == hidden_size and self.layers == [0]
        self.projs = nn.ModuleList([nn.Identity() if identity else nn.Linear(config.dim, hidden_size, bias=False)
                                    for _ in self.layers])
        # set by lazy (sparse-update) training: maps stacked row ids to the rows' values
        self.row_source: Callable[[torch.Tensor], torch.Tensor] | None = None

    @property
    def context(self) -> int:
        return max(self.orders) - 1

    def padded_tokens(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None) -> torch.Tensor:
        """``input_ids`` with ``context`` columns of left context in front (the end of
        ``prefix_ids`` where given, else the sentinel id)."""
        ctx = self.context
        left = input_ids.new_full((input_ids.shape[0], ctx), self.sentinel)
        if prefix_ids is not None and prefix_ids.shape[1]:
            keep = prefix_ids[:, -ctx:]
            left[:, ctx - keep.shape[1]:] = keep
        return torch.cat([left, input_ids], dim=1)

    def row_ids(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None = None) -> torch.Tensor:
        """(orders, batch, seq) row ids into the stacked tables."""
        tokens = self.padded_tokens(input_ids, prefix_ids)
        return torch.stack([ngram_bucket_ids(tokens, n, self.context, self.num_buckets) + k * self.num_buckets
                            for k, n in enumerate(self.orders)])

    def lookup(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None) -> torch.Tensor:
        if self.row_source is not None:
            return self.row_source(self.row_ids(input_ids, prefix_ids))
        if input_ids.is_cuda:
            weights = [t.weight for t in self.tables]
            return _NgramEmbed.apply(self.padded_tokens(input_ids, prefix_ids), self.context, tuple(self.orders),
                                     *weights)
        ids = self.row_ids(input_ids, prefix_ids)
        shards = getattr(self.tables[0].weight, "_mykb_table", None)  # row-sharded (parallel/sharded.py)
        if shards is not None:
            return shards.lookup_cpu(ids)
        return sum(t(ids[k] - k * self.num_buckets) for k, t in enumerate(self.tables))

    def forward(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None) -> dict[int, torch.Tensor]:
        feats = self.lookup(input_ids, prefix_ids)
        return {layer: (ops.linear(feats, proj.weight) if isinstance(proj, nn.Linear) else feats)
                for layer, proj in zip(self.layers, self.projs)}


class Embeddings(nn.Module):
    """Token embedding plus the optional n-gram embedding; ``forward`` returns the token
    rows and ``{block index: update}`` for the n-gram injections."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.token = nn.Embedding(config.vocab_size, config.hidden_size)
        self.ngram = NgramEmbedding(config.ngram, config.vocab_size, config.hidden_size) \
            if config.ngram.orders else None

    @property
    def context(self) -> int:
        return 0 if self.ngram is None else self.ngram.context

    def forward(self, input_ids: torch.Tensor, prefix_ids: torch.Tensor | None = None):
        injections = {} if self.ngram is None else self.ngram(input_ids, prefix_ids)
        return ops.embedding(input_ids, self.token.weight), injections
