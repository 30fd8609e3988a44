"""Pre-tokenised token shards: the reproducible data path for real runs.

On-disk format (identical to the reference's, ``src/myk_llm/data/shards.py:3-13``, so
shard sets are shared between the two):

    meta.json             {"tokenizer", "eos_id", "num_tokens", "token_dtype", "shards": [...]}
    shard_00000.bin       uint32 token ids, each document followed by the EOS id
    shard_00000.docs.npy  int64 exclusive end offset of every document in the shard

Reading is deterministic: each source is cut into windows of ``seq_len + 1`` tokens,
permuted per (seed, source, epoch); sources interleave by taking the one that has
consumed the fewest windows relative to its weight; every rank walks the same global
window sequence and keeps its slice.  The only state is a cursor per source, so a run
resumes exactly, also on a different number of GPUs.  A background thread prepares and
pins the next batches.
"""

from __future__ import annotations

import json
import queue
import threading
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Iterator

import numpy as np

from .config import IGNORE_INDEX, Batch, DataConfig, SourceConfig, collate

TOKEN_DTYPE = np.uint32


class ShardWriter:
    """Appends documents into fixed-size shards."""

    def __init__(self, directory, eos_id: int, tokenizer: str, shard_tokens: int = 1 << 28, prefix: str = "shard"):
        self.directory = Path(directory)
        self.directory.mkdir(parents=True, exist_ok=True)
        if (self.directory / "meta.json").exists():
            raise FileExistsError(f"{self.directory} already holds a shard set")
        self.eos_id, self.tokenizer, self.shard_tokens, self.prefix = eos_id, tokenizer, shard_tokens, prefix
        self.shards: list[dict[str, Any]] = []
        self._buf: list[np.ndarray] = []
        self._ends: list[int] = []
        self._n = 0

    @property
    def num_tokens(self) -> int:
        return sum(s["num_tokens"] for s in self.shards) + self._n

    def add(self, ids: list[int]) -> None:
        doc = np.asarray([*ids, self.eos_id], dtype=TOKEN_DTYPE)
        self._buf.append(doc)
        self._n += len(doc)
        self._ends.append(self._n)
        if self._n >= self.shard_tokens:
            self._flush()

    def _flush(self) -> None:
        if not self._n:
            return
        name = f"{self.prefix}_{len(self.shards):05d}"
        np.concatenate(self._buf).tofile(self.directory / f"{name}.bin")
        np.save(self.directory / f"{name}.docs.npy", np.asarray(self._ends, dtype=np.int64))
        self.shards.append({"file": f"{name}.bin", "num_tokens": self._n, "num_docs": len(self._ends)})
        self._buf, self._ends, self._n = [], [], 0

    def close(self, extra_meta: dict[str, Any] | None = None, write_meta: bool = True) -> list[dict[str, Any]]:
        self._flush()
        if write_meta:
            write_meta_file(self.directory, self.shards, self.eos_id, self.tokenizer, extra_meta)
        return self.shards


def write_meta_file(directory: Path, shards, eos_id: int, tokenizer: str, extra_meta=None) -> None:
    meta = {"tokenizer": tokenizer, "eos_id": eos_id, "num_tokens": sum(s["num_tokens"] for s in shards),
            "token_dtype": "uint32", "shards": shards, **(extra_meta or {})}
    (Path(directory) / "meta.json").write_text(json.dumps(meta, indent=2, ensure_ascii=False), encoding="utf-8")


class ShardSource:
    """Random access to one shard set as windows of seq_len + 1 tokens."""

    def __init__(self, config: SourceConfig, seq_len: int) -> None:
        self.config = config
        self.directory = Path(config.path)
        self.meta = json.loads((self.directory / "meta.json").read_text(encoding="utf-8"))
        self.seq_len = seq_len
        self._tokens: dict[int, np.ndarray] = {}
        self._ends: dict[int, np.ndarray] = {}
        ids, starts = [], []
        for i, sh in enumerate(self.meta["shards"]):
            count = max(0, (sh["num_tokens"] - 1) // seq_len)
            ids.append(np.full(count, i, dtype=np.int32))
            starts.append(np.arange(count, dtype=np.int64) * seq_len)
        self.window_shard = np.concatenate(ids) if ids else np.zeros(0, np.int32)
        self.window_start = np.concatenate(starts) if starts else np.zeros(0, np.int64)
        if len(self.window_shard) == 0:
            raise ValueError(f"{self.directory}: no complete window of {seq_len + 1} tokens")

    @property
    def eos_id(self) -> int:
        return int(self.meta["eos_id"])

    def __len__(self) -> int:
        return len(self.window_shard)

    def _shard(self, i: int):
        if i not in self._tokens:
            sh = self.meta["shards"][i]
            self._tokens[i] = np.memmap(self.directory / sh["file"], dtype=TOKEN_DTYPE, mode="r",
                                        shape=(sh["num_tokens"],))
            self._ends[i] = np.load(self.directory / sh["file"].replace(".bin", ".docs.npy"))
        return self._tokens[i], self._ends[i]

    def window(self, index: int, document_masking: bool) -> dict[str, np.ndarray]:
        toks, ends = self._shard(int(self.window_shard[index]))
        lo = int(self.window_start[index])
        hi = lo + self.seq_len
        chunk = np.asarray(toks[lo:hi + 1], dtype=np.int64)
        row = {"input_ids": chunk[:-1], "targets": chunk[1:].copy()}
        if document_masking:
            cuts = ends[np.searchsorted(ends, lo, side="right"):np.searchsorted(ends, hi, side="left")]
            row["targets"][cuts - lo - 1] = IGNORE_INDEX
            row["seqlens"] = np.diff(np.concatenate(([lo], cuts, [hi]))).astype(np.int32)
        return row


@dataclass
class _Cursor:
    epoch: int = 0
    position: int = 0
    consumed: int = 0


class ShardLoader:
    """Deterministic, resumable, rank-sliced batches over weighted shard sets."""

    def __init__(self, config: DataConfig, rank: int = 0, world_size: int = 1, prefetch: int = 4) -> None:
        if not config.sources:
            raise ValueError("data.sources is empty")
        self.config, self.rank, self.world_size = config, rank, world_size
        self.sources = [ShardSource(s, config.seq_len) for s in config.sources]
        self.weights = np.asarray([s.weight for s in config.sources], dtype=np.float64)
        if np.any(self.weights <= 0):
            raise ValueError("source weights must be positive")
        self.cursors = [_Cursor() for _ in self.sources]
        self._perm: dict[tuple[int, int], np.ndarray] = {}
        self.prefetch = prefetch
        self._queue: queue.Queue | None = None
        self._thread: threading.Thread | None = None
        self._stop = threading.Event()
        self._consumed_state: list[dict[str, int]] | None = None

    def _order(self, src: int, epoch: int) -> np.ndarray:
        key = (src, epoch)
        if key not in self._perm:
            if len(self._perm) > 2 * len(self.sources):
                self._perm.clear()
            rng = np.random.default_rng([self.config.seed, src, epoch])
            self._perm[key] = rng.permutation(len(self.sources[src]))
        return self._perm[key]

    def _next_window(self) -> tuple[int, int]:
        used = np.asarray([c.consumed for c in self.cursors], dtype=np.float64)
        src = int(np.argmin(used / self.weights))
        cur = self.cursors[src]
        order = self._order(src, cur.epoch)
        win = int(order[cur.position])
        cur.position += 1
        cur.consumed += 1
        if cur.position == len(order):
            cur.epoch, cur.position = cur.epoch + 1, 0
        return src, win

    def next_batch(self) -> Batch:
        per = self.config.micro_batch_size
        picks = [self._next_window() for _ in range(per * self.world_size)]
        mine = picks[self.rank * per:(self.rank + 1) * per]
        return collate([self.sources[s].window(w, self.config.document_masking) for s, w in mine])

    def __iter__(self) -> Iterator[Batch]:
        self._start()
        assert self._queue is not None
        while True:
            item = self._queue.get()
            if isinstance(item, BaseException):
                raise item
            batch, state = item
            self._consumed_state = state
            yield batch

    def _start(self) -> None:
        if self._thread is not None:
            return
        self._queue = queue.Queue(maxsize=self.prefetch)
        self._consumed_state = self._snapshot()

        def work() -> None:
            try:
                while not self._stop.is_set():
                    b = self.next_batch()
                    try:
                        b = b.pin_memory()
                    except RuntimeError:
                        pass  # no CUDA: plain host memory
                    self._queue.put((b, self._snapshot()))
            except BaseException as err:  # surface loader errors in the training loop
                self._queue.put(err)

        self._thread = threading.Thread(target=work, daemon=True, name="shard-loader")
        self._thread.start()

    def _snapshot(self) -> list[dict[str, int]]:
        return [vars(c).copy() for c in self.cursors]

    def state_dict(self) -> dict[str, Any]:
        cursors = self._consumed_state if self._thread is not None else self._snapshot()
        return {"kind": "shards", "cursors": cursors}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        if self._thread is not None:
            raise RuntimeError("load_state_dict must be called before iterating")
        self.cursors = [_Cursor(**c) for c in state["cursors"]]

    def close(self) -> None:
        self._stop.set()
