"""Data loaders.

Every loader yields this rank's ``Batch``es (pinned host memory, inputs and targets in one
tensor) and has ``state_dict`` / ``load_state_dict`` for an exact resume.  ``data.kind``
selects one: ``shards`` (pre-tokenised token shards), ``stream`` (tokenise while reading),
``sft`` (tokenised chat sets) or ``synthetic`` (packed random documents, the benchmarks'
source).  The reference's entry points of the same names are
``src/myk_llm/data/__init__.py:23-53``.
"""

from __future__ import annotations

from dataclasses import replace
from pathlib import Path
from typing import Any, Callable

from .config import IGNORE_INDEX, Batch, DataConfig, RowPacker, SourceConfig, SyntheticDataConfig, collate
from .filters import DocFilter


def resolve_eos_id(config: DataConfig) -> int:
    """Id of ``config.eos_token`` in the tokenizer at ``config.tokenizer``."""
    from tokenizers import Tokenizer

    vocab = Tokenizer.from_file(str(Path(config.tokenizer) / "tokenizer.json"))
    eos = vocab.token_to_id(config.eos_token)
    if eos is None:
        raise ValueError(f"eos_token {config.eos_token!r} is not in the tokenizer vocab")
    return int(eos)


def _shards(config: DataConfig, rank: int, world: int):
    from .shards import ShardLoader

    return ShardLoader(config, rank, world)


def _stream(config: DataConfig, rank: int, world: int):
    from .streaming import StreamLoader

    return StreamLoader(config, resolve_eos_id(config), rank, world)


def _sft(config: DataConfig, rank: int, world: int):
    from .sft import ChatLoader

    return ChatLoader(config, rank, world)


def _synthetic(config: DataConfig, rank: int, world: int):
    from .synthetic import SyntheticLoader

    return SyntheticLoader(config, rank, world)


LOADERS: dict[str, Callable[[DataConfig, int, int], Any]] = {
    "shards": _shards, "stream": _stream, "sft": _sft, "synthetic": _synthetic}


def build_loader(config: DataConfig, rank: int = 0, world_size: int = 1) -> Any:
    try:
        make = LOADERS[config.kind]
    except KeyError:
        raise ValueError(f"unknown data kind {config.kind!r}") from None
    return make(config, rank, world_size)


def build_fixed_batches(config: DataConfig, num_batches: int, seed: int) -> list[Batch]:
    """A fixed validation set: ``num_batches`` batches of ``micro_batch_size`` rows drawn
    with ``seed``, the same on every rank (ranks split the list, not the rows)."""
    if config.kind == "stream":
        from .streaming import take_windows

        rows = take_windows(config, resolve_eos_id(config), num_batches * config.micro_batch_size, seed)
        n = config.micro_batch_size
        return [collate(rows[i:i + n]) for i in range(0, num_batches * n, n)]
    loader = build_loader(replace(config, seed=seed), rank=0, world_size=1)
    if config.kind == "shards":  # a stateful order: consecutive batches
        return [loader.next_batch() for _ in range(num_batches)]
    return [loader.batch_at(i) for i in range(num_batches)]  # step-indexed sources


__all__ = ["IGNORE_INDEX", "LOADERS", "Batch", "DataConfig", "DocFilter", "RowPacker", "SourceConfig",
           "SyntheticDataConfig", "build_fixed_batches", "build_loader", "collate", "resolve_eos_id"]
