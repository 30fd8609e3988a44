"""Data configuration and the batch type.

``SourceConfig`` / ``DataConfig`` keep the reference's YAML schema
(``src/myk_llm/data/config.py:15-48``).  One extension: ``kind: synthetic`` with a
``synthetic`` sub-section, the packed random-document source used by the benchmarks.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

import numpy as np
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
    # Assign the rows of each global batch to ranks so that every rank gets about the same
    # attention work (sum of squared document lengths) instead of a fixed slice; the global
    # batch, and so the data-parallel gradient, is unchanged.
    balance_ranks: bool = False


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
    """One rank's micro-batch on the host (or, after ``to``, on the device).  Loaders that
    build batches with ``RowPacker`` keep inputs and targets in one pinned ``(2, B, S)``
    tensor (``staged``), so moving a batch to the GPU is a single asynchronous copy."""

    input_ids: torch.Tensor  # (batch, seq) int64
    targets: torch.Tensor  # (batch, seq) int64, IGNORE_INDEX where unsupervised
    seqlens: list[torch.Tensor] | None = None  # per-row document lengths (int32)
    staged: torch.Tensor | None = None

    def to(self, device: torch.device) -> "Batch":
        if self.staged is not None and torch.device(device).type == "cuda":
            both = self.staged.to(device, non_blocking=True)
            return Batch(both[0], both[1], self.seqlens)
        return Batch(self.input_ids.to(device, non_blocking=True), self.targets.to(device, non_blocking=True),
                     self.seqlens)

    def pin_memory(self) -> "Batch":
        if self.staged is not None and self.staged.is_pinned():
            return self
        both = torch.stack([self.input_ids, self.targets]).pin_memory()
        return Batch(both[0], both[1], self.seqlens, both)

    @property
    def num_targets(self) -> int:
        return int(torch.count_nonzero(self.targets != IGNORE_INDEX))

    @property
    def nbytes(self) -> int:
        return 2 * self.input_ids.numel() * self.input_ids.element_size()


def _pinned_ok() -> bool:
    return torch.cuda.is_available()


class RowPacker:
    """Writes the rows of one batch straight into a pinned host tensor: row ``i`` is a
    window of ``seq_len + 1`` tokens; its inputs are the first ``seq_len``, its targets the
    last ``seq_len`` with ``IGNORE_INDEX`` where ``ignore`` is set.  Document cut points
    (offsets inside the window where a document ends) become per-row ``seqlens``.  Pinned
    blocks come from torch's caching host allocator, which does not hand a block out again
    while an asynchronous copy from it may still be running."""

    def __init__(self, rows: int, seq_len: int, pin: bool | None = None) -> None:
        pin = _pinned_ok() if pin is None else pin
        self.seq_len = seq_len
        self.host = torch.empty((2, rows, seq_len), dtype=torch.long, pin_memory=pin)
        self.view = self.host.numpy()
        self.seqlens: list[torch.Tensor] = []
        self.masked = False

    def put(self, i: int, window: np.ndarray, ignore: np.ndarray | None = None,
            cuts: np.ndarray | None = None) -> None:
        self.view[0, i] = window[:-1]
        self.view[1, i] = window[1:]
        if ignore is not None:
            self.view[1, i][ignore] = IGNORE_INDEX
        if cuts is not None:
            self.masked = True
            bounds = np.concatenate(([0], np.asarray(cuts, dtype=np.int64), [self.seq_len]))
            self.seqlens.append(torch.from_numpy(np.diff(bounds).astype(np.int32)))

    def batch(self) -> Batch:
        return Batch(self.host[0], self.host[1], self.seqlens if self.masked else None, self.host)


def collate(rows: list[dict], pin: bool | None = None) -> Batch:
    """Batch from row dicts (``input_ids``, ``targets``, optional ``seqlens``).  Data-loader
    worker processes pass ``pin=False`` (a forked worker must not touch CUDA)."""
    packer = RowPacker(len(rows), len(rows[0]["input_ids"]), pin)
    for i, r in enumerate(rows):
        packer.view[0, i] = r["input_ids"]
        packer.view[1, i] = r["targets"]
        if "seqlens" in r:
            packer.masked = True
            packer.seqlens.append(torch.as_tensor(np.asarray(r["seqlens"], dtype=np.int32)))
    return packer.batch()
