"""Data configuration and the batch type.

``SourceConfig`` / ``DataConfig`` keep the reference's YAML schema
(``src/myk_llm/data/config.py:15-48``).  One extension: ``kind: synthetic`` with a
``synthetic`` sub-section, the packed random-document source used by the benchmarks.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

import torch

from .filters import DocFilter

IGNORE_INDEX = -100


@dataclass
class SourceConfig:
    name: str
    weight: float = 1.0
    path: str = ""
    hf_path: str = ""
    hf_config: str | None = None
    hf_data_dir: str | None = None
    hf_split: str = "train"
    text_key: str = "text"
    script: Literal["latin", "cjk"] | None = None
    curated: bool = False


@dataclass
class SyntheticDataConfig:
    """Packed synthetic documents: lengths ~ geometric(mean_doc_len) capped at seq_len,
    token ids uniform in [0, vocab_size) (skipping eos_id), EOS after every document."""

    vocab_size: int = 65536
    mean_doc_len: int = 1024
    eos_id: int = 0


@dataclass
class DataConfig:
    kind: Literal["shards", "stream", "sft", "synthetic"] = "shards"
    tokenizer: str = "_download_models/Qwen3.5-0.8B-pruned64k"
    seq_len: int = 2048
    micro_batch_size: int = 16
    sources: list[SourceConfig] = field(default_factory=list)
    document_masking: bool = True
    seed: int = 0
    eos_token: str = "<|endoftext|>"
    shuffle_buffer: int = 10_000
    num_workers: int = 4
    doc_filter: DocFilter = field(default_factory=DocFilter)
    synthetic: SyntheticDataConfig = field(default_factory=SyntheticDataConfig)


@dataclass
class Batch:
    input_ids: torch.Tensor  # (batch, seq) int64
    targets: torch.Tensor  # (batch, seq) int64, IGNORE_INDEX where unsupervised
    seqlens: list[torch.Tensor] | None = None  # per-row document lengths

    def to(self, device: torch.device) -> "Batch":
        return Batch(self.input_ids.to(device, non_blocking=True), self.targets.to(device, non_blocking=True),
                     self.seqlens)

    def pin_memory(self) -> "Batch":
        return Batch(self.input_ids.pin_memory(), self.targets.pin_memory(), self.seqlens)

    @property
    def num_targets(self) -> int:
        return int((self.targets != IGNORE_INDEX).sum())

    @property
    def nbytes(self) -> int:
        return self.input_ids.numel() * self.input_ids.element_size() + self.targets.numel() * self.targets.element_size()


def collate(rows: list[dict]) -> Batch:
    import numpy as np

    ids = torch.as_tensor(np.stack([r["input_ids"] for r in rows]), dtype=torch.long)
    tg = torch.as_tensor(np.stack([r["targets"] for r in rows]), dtype=torch.long)
    seqlens = [torch.as_tensor(r["seqlens"], dtype=torch.int32) for r in rows] if "seqlens" in rows[0] else None
    return Batch(ids, tg, seqlens)
