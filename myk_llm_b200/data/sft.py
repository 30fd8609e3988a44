"""Supervised fine-tuning data: chat transcripts with an assistant-only loss mask.

Files of a tokenised chat set with prefix ``P`` (an interface shared with the reference,
``src/myk_llm/data/sft.py:1-13``): ``P.tokens.bin`` (uint32 ids, conversations back to
back), ``P.loss_mask.bin`` (uint8, 1 where the token is supervised: assistant content and
its end-of-turn), ``P.spans.npy`` (int64 ``[start, end)`` per conversation) and
``P.meta.json``.

Training windows start at positions drawn from ``default_rng([seed, step])`` over the
whole token array, so conversations are packed rather than padded and the loader's only
state is the step; with document masking the conversation ends inside a window cut it.
Batches are assembled straight into pinned host memory (``RowPacker``).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Iterable, Iterator

import numpy as np

from .config import Batch, DataConfig, RowPacker

# role spellings of the two accepted transcript schemas, folded to chat-template roles
_ROLES = {"human": "user", "user": "user", "gpt": "assistant", "bot": "assistant", "assistant": "assistant",
          "system": "system"}
# (list key, role key, text key) of the accepted schemas: OpenAI-style and ShareGPT
_SCHEMAS = (("messages", "role", "content"), ("conversations", "from", "value"))


def normalize_messages(example: dict[str, Any]) -> list[dict[str, str]]:
    """``{"messages": [{"role", "content"}]}`` or ShareGPT ``{"conversations": [{"from",
    "value"}]}`` as a list of ``{"role", "content"}`` with canonical role names."""
    for list_key, role_key, text_key in _SCHEMAS:
        turns = example.get(list_key)
        if turns is None:
            continue
        if not isinstance(turns, list) or not turns:
            break
        out = []
        for turn in turns:
            role = turn.get(role_key, turn.get("role", turn.get("from")))
            text = turn.get(text_key, turn.get("content", turn.get("value")))
            if not (isinstance(role, str) and isinstance(text, str)):
                raise ValueError("chat messages need string role/content (or from/value)")
            out.append({"role": _ROLES.get(role.lower(), role), "content": text})
        return out
    raise ValueError("chat examples need a non-empty 'messages' or 'conversations' list")


def encode_chat(tokenizer, messages: list[dict[str, str]]) -> tuple[np.ndarray, np.ndarray]:
    """Token ids (uint32) and loss mask (uint8) from a chat template whose assistant turns
    are wrapped in ``{% generation %}`` (which is what makes the mask exact)."""
    enc = tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=False, return_dict=True,
                                        return_assistant_tokens_mask=True)
    ids = np.asarray(enc["input_ids"], dtype=np.uint32)
    mask = enc.get("assistant_masks")
    if mask is None or len(mask) != ids.size or ids.size == 0:
        raise ValueError("the chat template did not produce an assistant mask ({% generation %} tags missing?)")
    return ids, np.asarray(mask, dtype=np.uint8)


class _Growing:
    """An append-only numpy array that doubles its storage."""

    def __init__(self, dtype) -> None:
        self.data = np.empty(1 << 16, dtype=dtype)
        self.size = 0

    def extend(self, values: np.ndarray) -> None:
        need = self.size + values.size
        if need > self.data.size:
            grown = np.empty(max(need, 2 * self.data.size), dtype=self.data.dtype)
            grown[:self.size] = self.data[:self.size]
            self.data = grown
        self.data[self.size:need] = values
        self.size = need

    def array(self) -> np.ndarray:
        return self.data[:self.size]


def write_chat_dataset(tokenizer, examples: Iterable[dict[str, Any]], prefix, tokenizer_path: str) -> dict[str, Any]:
    """Tokenise transcripts into the chat-set files; conversations with fewer than two
    tokens or no supervised token are skipped and counted.  Returns the meta record."""
    toks, mask = _Growing(np.uint32), _Growing(np.uint8)
    spans: list[tuple[int, int]] = []
    skipped = 0
    for example in examples:
        ids, m = encode_chat(tokenizer, normalize_messages(example))
        if ids.size < 2 or not m.any():
            skipped += 1
            continue
        spans.append((toks.size, toks.size + ids.size))
        toks.extend(ids)
        mask.extend(m)
    return write_chat_arrays(prefix, toks.array(), mask.array(), spans, tokenizer_path, skipped)


def write_chat_arrays(prefix, toks, mask, spans, tokenizer_path: str = "", skipped: int = 0) -> dict[str, Any]:
    prefix = Path(prefix)
    prefix.parent.mkdir(parents=True, exist_ok=True)
    toks = np.asarray(toks, dtype=np.uint32)
    np.ascontiguousarray(toks).tofile(f"{prefix}.tokens.bin")
    np.ascontiguousarray(np.asarray(mask, dtype=np.uint8)).tofile(f"{prefix}.loss_mask.bin")
    np.save(f"{prefix}.spans.npy", np.asarray(spans, dtype=np.int64).reshape(-1, 2))
    meta = {"mode": "chat", "tokenizer": tokenizer_path, "num_tokens": int(toks.size), "num_spans": len(spans),
            "token_dtype": "uint32", "has_loss_mask": True, "skipped": skipped}
    Path(f"{prefix}.meta.json").write_text(json.dumps(meta, indent=2), encoding="utf-8")
    return meta


class ChatDataset:
    """Memory-mapped chat set."""

    def __init__(self, prefix) -> None:
        meta = json.loads(Path(f"{prefix}.meta.json").read_text(encoding="utf-8"))
        if not meta.get("has_loss_mask"):
            raise ValueError(f"{prefix} has no loss mask; tokenize it as chat data")
        n = self.num_tokens = int(meta["num_tokens"])
        self.tokens = np.memmap(f"{prefix}.tokens.bin", dtype=np.uint32, mode="r", shape=(n,))
        self.loss_mask = np.memmap(f"{prefix}.loss_mask.bin", dtype=np.uint8, mode="r", shape=(n,))
        self.doc_ends = np.load(f"{prefix}.spans.npy")[:, 1]

    def fill(self, packer: RowPacker, row: int, start: int, document_masking: bool) -> None:
        """Window of ``seq_len + 1`` tokens at ``start`` into a batch row: targets are the
        supervised next tokens only; conversation ends inside the window cut it."""
        seq = packer.seq_len
        chunk = np.asarray(self.tokens[start:start + seq + 1], dtype=np.int64)
        unsupervised = self.loss_mask[start + 1:start + seq + 1] == 0
        cuts = None
        if document_masking:
            e = self.doc_ends
            cuts = e[np.searchsorted(e, start, side="right"):np.searchsorted(e, start + seq, side="left")] - start
        packer.put(row, chunk, ignore=unsupervised, cuts=cuts)


class ChatLoader:
    """SFT batches for this rank; the state is the step counter."""

    def __init__(self, config: DataConfig, rank: int = 0, world_size: int = 1) -> None:
        if len(config.sources) != 1 or not config.sources[0].path:
            raise ValueError("sft data takes exactly one source with a tokenized `path` prefix")
        self.config, self.rank, self.world_size = config, rank, world_size
        self.dataset = ChatDataset(config.sources[0].path)
        if self.dataset.num_tokens < config.seq_len + 1:
            raise ValueError("chat dataset is shorter than one window")
        self.step = 0

    def batch_at(self, step: int) -> Batch:
        per, seq = self.config.micro_batch_size, self.config.seq_len
        starts = np.random.default_rng([self.config.seed, step]).integers(
            0, self.dataset.num_tokens - seq, size=per * self.world_size)
        packer = RowPacker(per, seq)
        for row, start in enumerate(starts[self.rank * per:(self.rank + 1) * per]):
            self.dataset.fill(packer, row, int(start), self.config.document_masking)
        return packer.batch()

    def next_batch(self) -> Batch:
        self.step += 1
        return self.batch_at(self.step - 1)

    def __iter__(self) -> Iterator[Batch]:
        while True:
            yield self.next_batch()

    def state_dict(self) -> dict[str, Any]:
        return {"kind": "sft", "step": self.step}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.step = int(state["step"])

    def close(self) -> None:
        pass
