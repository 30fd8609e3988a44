"""Pre-tokenised token shards: the reproducible data path for real runs.

On-disk format (an interface shared with the reference, ``src/myk_llm/data/shards.py:3-13``,
so shard sets are prepared once for both frameworks):

    meta.json             {"tokenizer", "eos_id", "num_tokens", "token_dtype": "uint32", "shards": [...]}
    shard_00000.bin       uint32 token ids, every document followed by the EOS id
    shard_00000.docs.npy  int64 exclusive end offset of every document within the shard

Window order (also shared, so a data-loader checkpoint resumes the same sequence in either
framework): a source of ``n`` windows of ``seq_len + 1`` tokens is visited in the order
``default_rng([seed, source, epoch]).permutation(n)``; the next window of the global
sequence comes from the source with the fewest windows taken relative to its weight; all
ranks walk that global sequence and each keeps its slice of every global batch.  The only
state is ``(epoch, position, consumed)`` per source.

This implementation locates windows arithmetically (a cumulative count per shard, no table
per window), memory-maps each shard once, and assembles every batch directly in a pinned
host tensor holding inputs and targets together (``RowPacker``), on a background thread,
so the trainer's host-to-device copy is one asynchronous transfer per batch.
"""

from __future__ import annotations

import json
import queue
import threading
from pathlib import Path
from typing import Any, Iterator

import numpy as np

from .config import Batch, DataConfig, RowPacker, SourceConfig

TOKEN_DTYPE = np.uint32
META = "meta.json"


def write_meta_file(directory: Path, shards: list[dict[str, Any]], eos_id: int, tokenizer: str,
                    extra_meta: dict[str, Any] | None = None) -> None:
    """meta.json for a list of shard records (also used to merge several writers' shards)."""
    meta = {"tokenizer": tokenizer, "eos_id": int(eos_id), "num_tokens": int(sum(r["num_tokens"] for r in shards)),
            "token_dtype": "uint32", "shards": list(shards)}
    meta.update(extra_meta or {})
    (Path(directory) / META).write_text(json.dumps(meta, indent=2, ensure_ascii=False), encoding="utf-8")


class ShardWriter:
    """Appends documents (each followed by EOS) into a growing uint32 buffer and writes a
    shard whenever it reaches ``shard_tokens``."""

    def __init__(self, directory, eos_id: int, tokenizer: str, shard_tokens: int = 1 << 28,
                 prefix: str = "shard") -> None:
        self.directory = Path(directory)
        self.directory.mkdir(parents=True, exist_ok=True)
        if (self.directory / META).exists():
            raise FileExistsError(f"{self.directory} already holds a shard set")
        self.eos_id, self.tokenizer, self.shard_tokens, self.prefix = int(eos_id), tokenizer, shard_tokens, prefix
        self.shards: list[dict[str, Any]] = []
        self._tokens = np.empty(1 << 16, dtype=TOKEN_DTYPE)
        self._fill = 0
        self._doc_ends: list[int] = []

    @property
    def num_tokens(self) -> int:
        return sum(r["num_tokens"] for r in self.shards) + self._fill

    def add(self, ids) -> None:
        doc = np.asarray(ids, dtype=TOKEN_DTYPE)
        need = self._fill + doc.size + 1
        if need > self._tokens.size:
            grown = np.empty(max(need, 2 * self._tokens.size), dtype=TOKEN_DTYPE)
            grown[:self._fill] = self._tokens[:self._fill]
            self._tokens = grown
        self._tokens[self._fill:self._fill + doc.size] = doc
        self._tokens[need - 1] = self.eos_id
        self._fill = need
        self._doc_ends.append(need)
        if self._fill >= self.shard_tokens:
            self._write_shard()

    def _write_shard(self) -> None:
        if self._fill == 0:
            return
        stem = f"{self.prefix}_{len(self.shards):05d}"
        self._tokens[:self._fill].tofile(self.directory / f"{stem}.bin")
        np.save(self.directory / f"{stem}.docs.npy", np.asarray(self._doc_ends, dtype=np.int64))
        self.shards.append({"file": f"{stem}.bin", "num_tokens": int(self._fill), "num_docs": len(self._doc_ends)})
        self._fill = 0
        self._doc_ends = []

    def close(self, extra_meta: dict[str, Any] | None = None, write_meta: bool = True) -> list[dict[str, Any]]:
        """Write the last shard and (unless several writers share the directory and merge
        their records with ``write_meta_file``) meta.json."""
        self._write_shard()
        if write_meta:
            write_meta_file(self.directory, self.shards, self.eos_id, self.tokenizer, extra_meta)
        return self.shards


class ShardSet:
    """One source directory seen as ``len(self)`` windows of ``seq_len + 1`` tokens; window
    ``w`` lives in shard ``searchsorted(first_window, w)`` at a multiple of ``seq_len``."""

    def __init__(self, config: SourceConfig, seq_len: int) -> None:
        self.config = config
        self.directory = Path(config.path)
        self.meta = json.loads((self.directory / META).read_text(encoding="utf-8"))
        self.seq_len = seq_len
        per_shard = np.asarray([max(0, (r["num_tokens"] - 1) // seq_len) for r in self.meta["shards"]], np.int64)
        self.first_window = np.concatenate(([0], np.cumsum(per_shard)))
        if self.first_window[-1] == 0:
            raise ValueError(f"{self.directory}: no complete window of {seq_len + 1} tokens")
        self._maps: dict[int, tuple[np.ndarray, np.ndarray]] = {}

    @property
    def eos_id(self) -> int:
        return int(self.meta["eos_id"])

    def __len__(self) -> int:
        return int(self.first_window[-1])

    def _open(self, shard: int) -> tuple[np.ndarray, np.ndarray]:
        got = self._maps.get(shard)
        if got is None:
            rec = self.meta["shards"][shard]
            toks = np.memmap(self.directory / rec["file"], dtype=TOKEN_DTYPE, mode="r", shape=(rec["num_tokens"],))
            ends = np.load(self.directory / (rec["file"][:-len(".bin")] + ".docs.npy"))
            got = self._maps[shard] = (toks, ends)
        return got

    def locate(self, window: int) -> tuple[int, int]:
        shard = int(np.searchsorted(self.first_window, window, side="right")) - 1
        return shard, int(window - self.first_window[shard]) * self.seq_len

    def fill(self, packer: RowPacker, row: int, window: int, document_masking: bool) -> None:
        """Write window ``window`` into row ``row`` of a batch being packed.  Document ends
        strictly inside the window cut it; the EOS that ends a document keeps its place and
        its target (the next document's first token) is masked."""
        shard, lo = self.locate(window)
        toks, ends = self._open(shard)
        hi = lo + self.seq_len
        chunk = np.asarray(toks[lo:hi + 1], dtype=np.int64)
        if not document_masking:
            packer.put(row, chunk)
            return
        inside = ends[np.searchsorted(ends, lo, side="right"):np.searchsorted(ends, hi, side="left")] - lo
        packer.put(row, chunk, ignore=inside - 1, cuts=inside)

    def window(self, window: int, document_masking: bool) -> dict[str, np.ndarray]:
        """One window as arrays (``input_ids``, ``targets``, and ``seqlens`` when masking)."""
        packer = RowPacker(1, self.seq_len, pin=False)
        self.fill(packer, 0, window, document_masking)
        row = {"input_ids": packer.view[0, 0].copy(), "targets": packer.view[1, 0].copy()}
        if document_masking:
            row["seqlens"] = packer.seqlens[0].numpy()
        return row


ShardSource = ShardSet  # the reference's name for the same role


class WindowOrder:
    """The deterministic global window sequence over weighted sources (see module
    docstring); ``cursors`` is the whole state."""

    def __init__(self, sizes: list[int], weights: list[float], seed: int) -> None:
        self.sizes = [int(n) for n in sizes]
        self.weights = np.asarray(weights, dtype=np.float64)
        if np.any(self.weights <= 0):
            raise ValueError("source weights must be positive")
        self.seed = seed
        self.cursors = [{"epoch": 0, "position": 0, "consumed": 0} for _ in sizes]
        self._perm_key: list[int | None] = [None] * len(sizes)
        self._perm: list[np.ndarray | None] = [None] * len(sizes)

    def _permutation(self, src: int, epoch: int) -> np.ndarray:
        if self._perm_key[src] != epoch:
            self._perm[src] = np.random.default_rng([self.seed, src, epoch]).permutation(self.sizes[src])
            self._perm_key[src] = epoch
        return self._perm[src]

    def take(self, count: int) -> list[tuple[int, int]]:
        """The next ``count`` (source, window) pairs; advances the cursors."""
        out = []
        consumed = np.asarray([c["consumed"] for c in self.cursors], dtype=np.float64)
        for _ in range(count):
            src = int(np.argmin(consumed / self.weights))
            cur = self.cursors[src]
            out.append((src, int(self._permutation(src, cur["epoch"])[cur["position"]])))
            consumed[src] += 1
            cur["consumed"] += 1
            cur["position"] += 1
            if cur["position"] == self.sizes[src]:
                cur["epoch"] += 1
                cur["position"] = 0
        return out

    def snapshot(self) -> list[dict[str, int]]:
        return [dict(c) for c in self.cursors]

    def restore(self, cursors: list[dict[str, int]]) -> None:
        if len(cursors) != len(self.sizes):
            raise ValueError(f"checkpoint has {len(cursors)} source cursors, the config {len(self.sizes)} sources")
        self.cursors = [{"epoch": int(c["epoch"]), "position": int(c["position"]), "consumed": int(c["consumed"])}
                        for c in cursors]


class ShardLoader:
    """Deterministic, resumable, rank-sliced batches over weighted shard sets; iterating
    runs a background thread that keeps ``prefetch`` pinned batches ready."""

    def __init__(self, config: DataConfig, rank: int = 0, world_size: int = 1, prefetch: int = 4) -> None:
        if not config.sources:
            raise ValueError("data.sources is empty")
        self.config, self.rank, self.world_size, self.prefetch = config, rank, world_size, prefetch
        self.sources = [ShardSet(s, config.seq_len) for s in config.sources]
        self.order = WindowOrder([len(s) for s in self.sources], [s.weight for s in config.sources], config.seed)
        self._ready: queue.Queue | None = None
        self._worker: threading.Thread | None = None
        self._halt = threading.Event()
        self._handed_out = self.order.snapshot()  # cursors after the last batch the trainer took

    def next_batch(self) -> Batch:
        """This rank's slice of the next global batch (advances the shared order)."""
        per = self.config.micro_batch_size
        picks = self.order.take(per * self.world_size)[self.rank * per:(self.rank + 1) * per]
        packer = RowPacker(per, self.config.seq_len)
        for row, (src, win) in enumerate(picks):
            self.sources[src].fill(packer, row, win, self.config.document_masking)
        return packer.batch()

    def __iter__(self) -> Iterator[Batch]:
        if self._worker is None:
            self._ready = queue.Queue(maxsize=self.prefetch)
            self._worker = threading.Thread(target=self._produce, daemon=True, name="shard-loader")
            self._worker.start()
        while True:
            item = self._ready.get()
            if isinstance(item, BaseException):
                raise item
            batch, self._handed_out = item
            yield batch

    def _produce(self) -> None:
        try:
            while not self._halt.is_set():
                batch = self.next_batch()
                self._ready.put((batch, self.order.snapshot()))
        except BaseException as err:  # surfaces in the training loop's next batch
            self._ready.put(err)

    def state_dict(self) -> dict[str, Any]:
        cursors = self._handed_out if self._worker is not None else self.order.snapshot()
        return {"kind": "shards", "cursors": [dict(c) for c in cursors]}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        if self._worker is not None:
            raise RuntimeError("load_state_dict must be called before iterating")
        self.order.restore(state["cursors"])
        self._handed_out = self.order.snapshot()

    def close(self) -> None:
        self._halt.set()
