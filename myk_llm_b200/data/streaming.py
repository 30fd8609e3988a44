"""Streaming corpus: documents read from HuggingFace ``datasets`` streams (a hub dataset,
or local json/jsonl/parquet/text files given as a source ``path``), tokenized on the fly
and packed into fixed windows.

Behaviour follows the reference's ``src/myk_llm/data/streaming.py:36-263``:

* every rank reads a disjoint part of every source (``split_dataset_by_node``), shuffled
  through a buffer; a source that runs out reshuffles with the next seed and loops;
* sources are interleaved by token budget: the next document comes from the source with
  the smallest consumed-tokens / weight ratio;
* documents are concatenated with an EOS after each; a window of ``seq_len + 1`` tokens
  gives inputs / targets; with ``document_masking`` each row carries its per-document
  lengths and targets that cross a document seam are masked;
* all iteration state (stream position, queued documents, the partial window) is plain
  data, so ``state_dict`` restores the stream exactly.

Pre-tokenized shards (``data.shards``) remain the path for long runs: they need no
tokenizer at load time and resume by cursor.
"""

from __future__ import annotations

import functools

import glob
from pathlib import Path
from typing import Any, Iterator

import numpy as np
from torch.utils.data import IterableDataset, get_worker_info

from .config import IGNORE_INDEX, Batch, DataConfig, SourceConfig, collate
from .filters import DocFilter

_LOCAL_BUILDERS = {".json": "json", ".jsonl": "json", ".parquet": "parquet", ".txt": "text", ".arrow": "arrow"}


def open_stream(source: SourceConfig, seed: int, shuffle_buffer: int, rank: int = 0, world_size: int = 1):
    """A shuffled, rank-split streaming ``datasets.IterableDataset`` of one source."""
    from datasets import load_dataset

    if source.path:
        files = sorted(glob.glob(source.path)) if any(c in source.path for c in "*?[") \
            else [source.path]
        if not files:
            raise FileNotFoundError(f"source {source.name!r}: no files match {source.path!r}")
        builder = _LOCAL_BUILDERS.get(Path(files[0]).suffix)
        if builder is None:
            raise ValueError(f"source {source.name!r}: unsupported file type {Path(files[0]).suffix!r}")
        ds = load_dataset(builder, data_files=files, split="train", streaming=True)
    else:
        ds = load_dataset(source.hf_path, name=source.hf_config, data_dir=source.hf_data_dir, split=source.hf_split,
                          streaming=True)
    if world_size > 1:
        from datasets.distributed import split_dataset_by_node

        ds = split_dataset_by_node(ds, rank=rank, world_size=world_size)
    if shuffle_buffer > 0:
        ds = ds.shuffle(seed=seed, buffer_size=shuffle_buffer)
    return ds


class TokenizedSource:
    """One source: raw documents -> filtered token lists (EOS appended), batched through
    the tokenizer, endless by reshuffling each epoch.  State = (epoch, the stream's own
    position, the queue of tokenized but unconsumed documents)."""

    def __init__(self, source: SourceConfig, tokenizer: Any, seed: int, shuffle_buffer: int, eos_id: int,
                 doc_filter: DocFilter, rank: int = 0, world_size: int = 1, encode_batch: int = 64,
                 open_fn=open_stream) -> None:
        self.source, self.tokenizer, self.seed, self.shuffle_buffer = source, tokenizer, seed, shuffle_buffer
        self.eos_id, self.doc_filter, self.rank, self.world_size = eos_id, doc_filter, rank, world_size
        self.encode_batch, self.open_fn = encode_batch, open_fn
        self.epoch = 0
        self.kept = self.dropped = self.dropped_text = 0
        self.queue: list[list[int]] = []
        self._ds = None
        self._it: Iterator[dict[str, Any]] | None = None
        self._resume: dict[str, Any] | None = None

    def _open(self) -> None:
        self._ds = self.open_fn(self.source, self.seed + self.epoch, self.shuffle_buffer, self.rank, self.world_size)
        if self._resume is not None:
            self._ds.load_state_dict(self._resume)
            self._resume = None
        self._it = iter(self._ds)

    def _texts(self) -> list[str]:
        if self._it is None:
            self._open()
        texts: list[str] = []
        while len(texts) < self.encode_batch:
            try:
                example = next(self._it)
            except StopIteration:
                self.epoch += 1
                self._open()
                continue
            text = example.get(self.source.text_key)
            if not isinstance(text, str) or not text.strip():
                continue
            if not self.source.curated and self.doc_filter.reject_text(text, self.source.script):
                self.dropped_text += 1
                continue
            texts.append(text)
        return texts

    def _refill(self) -> None:
        cap = self.doc_filter.max_doc_tokens
        for enc in self.tokenizer.encode_batch(self._texts(), add_special_tokens=False):
            ids = list(enc.ids)
            if not ids:
                continue
            if cap and len(ids) > cap:
                ids = ids[:cap]
            if not self.source.curated and self.doc_filter.reject(ids):
                self.dropped += 1
                continue
            self.kept += 1
            ids.append(self.eos_id)
            self.queue.append(ids)

    def next_doc(self) -> list[int]:
        while not self.queue:
            self._refill()
        return self.queue.pop(0)

    def state_dict(self) -> dict[str, Any]:
        if self._it is None:
            self._open()
        return {"epoch": self.epoch, "queue": [list(d) for d in self.queue], "stream": self._ds.state_dict()}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.epoch = int(state.get("epoch", 0))
        self.queue = [list(d) for d in state.get("queue", [])]
        self._resume = state.get("stream")
        self._it = None


class Packer:
    """Token-balanced interleave of sources packed into windows of seq_len + 1 tokens."""

    def __init__(self, sources: list[Any], weights: list[float], seq_len: int, document_masking: bool) -> None:
        self.sources, self.seq_len, self.masking = sources, seq_len, document_masking
        self.weights = np.asarray(weights, dtype=np.float64)
        self.consumed = np.zeros(len(sources), dtype=np.float64)
        self.tokens: list[int] = []
        self.segments: list[int] = []
        self.next_segment = 0

    def window(self) -> dict[str, np.ndarray]:
        n = self.seq_len + 1
        while len(self.tokens) < n:
            k = int(np.argmin(self.consumed / self.weights))
            doc = self.sources[k].next_doc()
            self.consumed[k] += len(doc)
            self.tokens.extend(doc)
            self.segments.extend([self.next_segment] * len(doc))
            self.next_segment += 1
        toks = np.asarray(self.tokens[:n], dtype=np.int64)
        segs = np.asarray(self.segments[:n], dtype=np.int64)
        # the last token of this window is the first of the next one
        del self.tokens[:self.seq_len], self.segments[:self.seq_len]
        row = {"input_ids": toks[:-1].copy(), "targets": toks[1:].copy()}
        if self.masking:
            seam = segs[:-1] != segs[1:]
            row["targets"][seam] = IGNORE_INDEX
            starts = np.flatnonzero(np.diff(segs[:-1])) + 1
            row["seqlens"] = np.diff(np.concatenate(([0], starts, [self.seq_len]))).astype(np.int32)
        return row

    def state_dict(self) -> dict[str, Any]:
        return {"consumed": self.consumed.tolist(), "tokens": list(self.tokens), "segments": list(self.segments),
                "next_segment": self.next_segment, "sources": [s.state_dict() for s in self.sources]}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.consumed = np.asarray(state["consumed"], dtype=np.float64)
        self.tokens, self.segments = list(state["tokens"]), list(state["segments"])
        self.next_segment = int(state["next_segment"])
        for src, st in zip(self.sources, state["sources"]):
            src.load_state_dict(st)


class PackedStreamDataset(IterableDataset):
    """Endless packed windows of this rank's share of ``config.sources``; each DataLoader
    worker decorrelates its shuffle seed by its worker id."""

    def __init__(self, config: DataConfig, eos_id: int, rank: int = 0, world_size: int = 1, seed: int | None = None,
                 tokenizer: Any = None, open_fn=open_stream) -> None:
        super().__init__()
        if not config.sources:
            raise ValueError("data.sources is empty")
        self.config, self.eos_id, self.rank, self.world_size = config, eos_id, rank, world_size
        self.seed = config.seed if seed is None else seed
        self.tokenizer, self.open_fn = tokenizer, open_fn
        self.packer: Packer | None = None
        self._pending: dict[str, Any] | None = None

    def _setup(self) -> None:
        if self.packer is not None:
            return
        worker = get_worker_info()
        seed = self.seed + 1009 * (worker.id if worker is not None else 0)
        tok = self.tokenizer
        if tok is None:
            from tokenizers import Tokenizer

            tok = Tokenizer.from_file(str(Path(self.config.tokenizer) / "tokenizer.json"))
        c = self.config
        sources = [TokenizedSource(s, tok, seed, c.shuffle_buffer, self.eos_id, c.doc_filter, self.rank,
                                   self.world_size, open_fn=self.open_fn) for s in c.sources]
        self.packer = Packer(sources, [s.weight for s in c.sources], c.seq_len, c.document_masking)
        if self._pending:
            self.packer.load_state_dict(self._pending)
        self._pending = None

    def __iter__(self) -> Iterator[dict[str, np.ndarray]]:
        self._setup()
        while True:
            yield self.packer.window()

    def state_dict(self) -> dict[str, Any]:
        return self.packer.state_dict() if self.packer is not None else (self._pending or {})

    def load_state_dict(self, state: dict[str, Any]) -> None:
        if self.packer is None:
            self._pending = state
        elif state:
            self.packer.load_state_dict(state)


class StreamLoader:
    """This rank's batches: torchdata's StatefulDataLoader over ``PackedStreamDataset``
    (its state covers every worker), collated into pinned ``Batch``es."""

    def __init__(self, config: DataConfig, eos_id: int, rank: int = 0, world_size: int = 1, **dataset_kw) -> None:
        from torchdata.stateful_dataloader import StatefulDataLoader

        workers = config.num_workers
        self.loader = StatefulDataLoader(
            PackedStreamDataset(config, eos_id, rank, world_size, **dataset_kw), batch_size=config.micro_batch_size,
            num_workers=workers, collate_fn=functools.partial(collate, pin=False), pin_memory=workers > 0, drop_last=True,
            persistent_workers=workers > 0, prefetch_factor=4 if workers > 0 else None)
        self._it: Iterator[Batch] | None = None

    def __iter__(self) -> Iterator[Batch]:
        return iter(self.loader)

    def next_batch(self) -> Batch:
        if self._it is None:
            self._it = iter(self.loader)
        return next(self._it)

    def state_dict(self) -> dict[str, Any]:
        return {"kind": "stream", "loader": self.loader.state_dict()}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.loader.load_state_dict(state["loader"])
        self._it = None

    def close(self) -> None:
        self._it = None


def take_windows(config: DataConfig, eos_id: int, num_rows: int, seed: int, **dataset_kw) -> list[dict[str, np.ndarray]]:
    """A fixed list of windows (a monitoring validation set) from a dedicated seed."""
    it = iter(PackedStreamDataset(config, eos_id, seed=seed, **dataset_kw))
    return [next(it) for _ in range(num_rows)]
