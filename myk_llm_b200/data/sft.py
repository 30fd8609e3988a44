"""Supervised fine-tuning data: chat transcripts with an assistant-only loss mask.

File layout (shared with the reference, ``src/myk_llm/data/sft.py:60-83``):
``P.tokens.bin`` (uint32), ``P.loss_mask.bin`` (uint8, 1 on assistant tokens),
``P.spans.npy`` (int64 [start, end) per conversation) and ``P.meta.json``.
``ChatLoader`` draws window starts from a generator seeded with (seed, step), so its
only state is the step.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Iterable, Iterator

import numpy as np

from .config import IGNORE_INDEX, Batch, DataConfig, collate

ROLE_ALIASES = {"human": "user", "user": "user", "gpt": "assistant", "assistant": "assistant", "bot": "assistant",
                "system": "system"}


def normalize_messages(example: dict[str, Any]) -> list[dict[str, str]]:
    """{'messages': [{role, content}]} or ShareGPT {'conversations': [{from, value}]}."""
    msgs = example.get("messages", example.get("conversations"))
    if not isinstance(msgs, list) or not msgs:
        raise ValueError("chat examples need a non-empty 'messages' or 'conversations' list")
    out = []
    for m in msgs:
        role, content = m.get("role", m.get("from")), m.get("content", m.get("value"))
        if not isinstance(role, str) or not isinstance(content, str):
            raise ValueError("chat messages need string role/content (or from/value)")
        out.append({"role": ROLE_ALIASES.get(role.lower(), role), "content": content})
    return out


def encode_chat(tokenizer, messages: list[dict[str, str]]) -> tuple[list[int], list[int]]:
    """Token ids and the assistant mask produced by a chat template with
    ``{% generation %}`` blocks."""
    enc = tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=False, return_dict=True,
                                        return_assistant_tokens_mask=True)
    ids = [int(t) for t in enc["input_ids"]]
    mask = enc.get("assistant_masks")
    if not mask or len(mask) != len(ids):
        raise ValueError("the chat template did not produce an assistant mask ({% generation %} tags missing?)")
    return ids, [int(m) for m in mask]


def write_chat_dataset(tokenizer, examples: Iterable[dict[str, Any]], prefix, tokenizer_path: str) -> dict[str, Any]:
    prefix = Path(prefix)
    prefix.parent.mkdir(parents=True, exist_ok=True)
    toks: list[int] = []
    mask: list[int] = []
    spans: list[tuple[int, int]] = []
    skipped = 0
    for ex in examples:
        ids, m = encode_chat(tokenizer, normalize_messages(ex))
        if len(ids) < 2 or not any(m):
            skipped += 1
            continue
        spans.append((len(toks), len(toks) + len(ids)))
        toks.extend(ids)
        mask.extend(m)
    write_chat_arrays(prefix, toks, mask, spans, tokenizer_path, skipped)
    return json.loads(Path(f"{prefix}.meta.json").read_text())


def write_chat_arrays(prefix, toks, mask, spans, tokenizer_path: str = "", skipped: int = 0) -> None:
    np.asarray(toks, dtype=np.uint32).tofile(f"{prefix}.tokens.bin")
    np.asarray(mask, dtype=np.uint8).tofile(f"{prefix}.loss_mask.bin")
    np.save(f"{prefix}.spans.npy", np.asarray(spans, dtype=np.int64).reshape(-1, 2))
    meta = {"mode": "chat", "tokenizer": tokenizer_path, "num_tokens": len(toks), "num_spans": len(spans),
            "token_dtype": "uint32", "has_loss_mask": True, "skipped": skipped}
    Path(f"{prefix}.meta.json").write_text(json.dumps(meta, indent=2), encoding="utf-8")


class ChatDataset:
    def __init__(self, prefix) -> None:
        meta = json.loads(Path(f"{prefix}.meta.json").read_text(encoding="utf-8"))
        if not meta.get("has_loss_mask"):
            raise ValueError(f"{prefix} has no loss mask; tokenize it as chat data")
        self.num_tokens = int(meta["num_tokens"])
        self.tokens = np.memmap(f"{prefix}.tokens.bin", dtype=np.uint32, mode="r", shape=(self.num_tokens,))
        self.loss_mask = np.memmap(f"{prefix}.loss_mask.bin", dtype=np.uint8, mode="r", shape=(self.num_tokens,))
        self.doc_ends = np.load(f"{prefix}.spans.npy")[:, 1]

    def window(self, start: int, seq_len: int, document_masking: bool) -> dict[str, np.ndarray]:
        chunk = np.asarray(self.tokens[start:start + seq_len + 1], dtype=np.int64)
        m = np.asarray(self.loss_mask[start + 1:start + seq_len + 1], dtype=bool)
        row = {"input_ids": chunk[:-1], "targets": np.where(m, chunk[1:], IGNORE_INDEX)}
        if document_masking:
            lo, hi = start, start + seq_len
            e = self.doc_ends
            cuts = e[np.searchsorted(e, lo, side="right"):np.searchsorted(e, hi, side="left")]
            row["seqlens"] = np.diff(np.concatenate(([lo], cuts, [hi]))).astype(np.int32)
        return row


class ChatLoader:
    def __init__(self, config: DataConfig, rank: int = 0, world_size: int = 1) -> None:
        if len(config.sources) != 1 or not config.sources[0].path:
            raise ValueError("sft data takes exactly one source with a tokenized `path` prefix")
        self.config, self.rank, self.world_size = config, rank, world_size
        self.dataset = ChatDataset(config.sources[0].path)
        if self.dataset.num_tokens < config.seq_len + 1:
            raise ValueError("chat dataset is shorter than one window")
        self.step = 0

    def batch_at(self, step: int) -> Batch:
        per = self.config.micro_batch_size
        rng = np.random.default_rng([self.config.seed, step])
        starts = rng.integers(0, self.dataset.num_tokens - self.config.seq_len, size=per * self.world_size)
        mine = starts[self.rank * per:(self.rank + 1) * per]
        return collate([self.dataset.window(int(s), self.config.seq_len, self.config.document_masking) for s in mine])

    def next_batch(self) -> Batch:
        b = self.batch_at(self.step)
        self.step += 1
        return b

    def __iter__(self) -> Iterator[Batch]:
        while True:
            yield self.next_batch()

    def state_dict(self) -> dict[str, Any]:
        return {"kind": "sft", "step": self.step}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.step = int(state["step"])

    def close(self) -> None:
        pass
