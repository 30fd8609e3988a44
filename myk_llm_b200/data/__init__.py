"""Data loaders.  Each yields ``Batch``es for this rank and has ``state_dict`` /
``load_state_dict`` for exact resume (reference: ``src/myk_llm/data/__init__.py:23-53``)."""

from __future__ import annotations

from pathlib import Path
from typing import Any

from .config import IGNORE_INDEX, Batch, DataConfig, SourceConfig, SyntheticDataConfig, collate
from .filters import DocFilter


def resolve_eos_id(config: DataConfig) -> int:
    from tokenizers import Tokenizer

    tok = Tokenizer.from_file(str(Path(config.tokenizer) / "tokenizer.json"))
    eos = tok.token_to_id(config.eos_token)
    if eos is None:
        raise ValueError(f"eos_token {config.eos_token!r} is not in the tokenizer vocab")
    return int(eos)


def build_loader(config: DataConfig, rank: int = 0, world_size: int = 1) -> Any:
    if config.kind == "shards":
        from .shards import ShardLoader

        return ShardLoader(config, rank, world_size)
    if config.kind == "stream":
        from .streaming import StreamLoader

        return StreamLoader(config, resolve_eos_id(config), rank, world_size)
    if config.kind == "sft":
        from .sft import ChatLoader

        return ChatLoader(config, rank, world_size)
    if config.kind == "synthetic":
        from .synthetic import SyntheticLoader

        return SyntheticLoader(config, rank, world_size)
    raise ValueError(f"unknown data kind {config.kind!r}")


def build_fixed_batches(config: DataConfig, num_batches: int, seed: int) -> list[Batch]:
    """A fixed validation set of ``num_batches`` global batches, identical on every rank."""
    from dataclasses import replace

    if config.kind == "stream":
        from .streaming import take_windows

        rows = take_windows(config, resolve_eos_id(config), num_batches * config.micro_batch_size, seed)
        n = config.micro_batch_size
        return [collate(rows[i * n:(i + 1) * n]) for i in range(num_batches)]
    loader = build_loader(replace(config, seed=seed), rank=0, world_size=1)
    if config.kind == "shards":
        return [loader.next_batch() for _ in range(num_batches)]
    return [loader.batch_at(i) for i in range(num_batches)]


__all__ = ["IGNORE_INDEX", "Batch", "DataConfig", "DocFilter", "SourceConfig", "SyntheticDataConfig",
           "build_fixed_batches", "build_loader", "collate", "resolve_eos_id"]
