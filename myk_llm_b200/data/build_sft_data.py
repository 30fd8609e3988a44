"""Assemble a chat (SFT) dataset as normalized JSONL from instruction sources.

Rows in any of three shapes are normalized to ``{"messages": [{role, content}, ...]}``:
``messages`` lists, ShareGPT ``conversations`` (from / value) and Alpaca-style
``instruction`` (+ ``input``) / ``output``.  Each source is streamed and capped,
length-filtered, deduplicated across sources (hash of the role:content sequence), then
the union is shuffled with a fixed seed and split into train / val JSONL (the pipeline
of the reference's ``scripts/build_sft_data.py``; its default source list is kept as
the default here)::

    python -m myk_llm_b200.data.build_sft_data --out-dir data/sft --max-per-source 200000 --val-frac 0.01
    python -m myk_llm_b200.data.build_sft_data --out-dir data/sft --source local:data/raw/*.jsonl
"""

from __future__ import annotations

import argparse
import glob
import hashlib
import json
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Iterable, Iterator

ROLES = {"human": "user", "user": "user", "gpt": "assistant", "assistant": "assistant", "bot": "assistant",
         "system": "system"}


@dataclass
class Source:
    name: str
    path: str                     # hub id, or local:<glob> for jsonl files
    configs: list[str | None] = field(default_factory=lambda: [None])
    split: str = "train"
    max_assistant_chars: int | None = None


DEFAULT_SOURCES = [
    Source("smoltalk", "HuggingFaceTB/smoltalk",
           ["smol-magpie-ultra", "smol-summarize", "smol-rewrite", "smol-constraints", "everyday-conversations",
            "systemchats-30k", "openhermes-100k", "explore-instruct-rewriting"]),
    Source("coig-cqia", "m-a-p/COIG-CQIA",
           ["coig_pc", "exam", "human_value", "logi_qa", "ruozhiba", "wiki", "wikihow", "zhihu", "xhs", "douban",
            "finance", "segmentfault"]),
    Source("finewebedu-zh", "opencsg/Fineweb-Edu-Chinese-V2.2", ["default"], split="sft_qa", max_assistant_chars=1200),
]


def _text(v: Any) -> str:
    return v.strip() if isinstance(v, str) else ""


def to_messages(row: dict[str, Any]) -> list[dict[str, str]] | None:
    raw = row.get("messages") or row.get("conversations")
    if isinstance(raw, list) and raw:
        msgs = []
        for m in raw:
            if not isinstance(m, dict):
                return None
            role, content = m.get("role", m.get("from")), _text(m.get("content", m.get("value")))
            if not isinstance(role, str) or not content:
                return None
            msgs.append({"role": ROLES.get(role.lower(), role), "content": content})
    else:
        ins, extra = _text(row.get("instruction")), _text(row.get("input"))
        out = _text(row.get("output") or row.get("response") or row.get("answer"))
        if not ins or not out:
            return None
        msgs = [{"role": "user", "content": f"{ins}\n\n{extra}" if extra else ins},
                {"role": "assistant", "content": out}]
    if not any(m["role"] == "assistant" for m in msgs) or (msgs[0]["role"] == "system" and len(msgs) < 2):
        return None
    return msgs


def keep(msgs: list[dict[str, str]], min_chars: int, max_chars: int, max_assistant: int | None) -> bool:
    total = sum(len(m["content"]) for m in msgs)
    if not min_chars <= total <= max_chars:
        return False
    asst = sum(len(m["content"]) for m in msgs if m["role"] == "assistant")
    return max_assistant is None or asst <= max_assistant


def dedup_key(msgs: list[dict[str, str]]) -> str:
    return hashlib.sha1("\x1f".join(f"{m['role']}:{m['content']}" for m in msgs).encode("utf-8")).hexdigest()


def rows_of(src: Source) -> Iterator[dict[str, Any]]:
    if src.path.startswith("local:"):
        for f in sorted(glob.glob(src.path[len("local:"):])):
            with open(f, encoding="utf-8") as fh:
                for line in fh:
                    if line.strip():
                        yield json.loads(line)
        return
    from datasets import load_dataset

    for cfg in src.configs:
        try:
            ds = load_dataset(src.path, name=cfg, split=src.split, streaming=True)
        except Exception as err:  # noqa: BLE001 - a gated or missing config is skipped, the rest go on
            print(f"  [warn] {src.name}:{cfg} unavailable ({type(err).__name__}); skipped")
            continue
        yield from ds


def collect(sources: Iterable[Source], cap: int, min_chars: int, max_chars: int) -> tuple[list, dict]:
    seen: set[str] = set()
    out, stats = [], {}
    for src in sources:
        n = 0
        for row in rows_of(src):
            if n >= cap:
                break
            msgs = to_messages(row)
            if msgs is None or not keep(msgs, min_chars, max_chars, src.max_assistant_chars):
                continue
            k = dedup_key(msgs)
            if k in seen:
                continue
            seen.add(k)
            out.append({"messages": msgs, "source": src.name})
            n += 1
        stats[src.name] = n
    return out, stats


def write_split(rows: list, out_dir: Path, val_frac: float, seed: int) -> dict:
    random.Random(seed).shuffle(rows)
    nval = int(len(rows) * val_frac)
    out_dir.mkdir(parents=True, exist_ok=True)
    for name, part in (("val", rows[:nval]), ("train", rows[nval:])):
        with (out_dir / f"{name}.jsonl").open("w", encoding="utf-8") as f:
            for r in part:
                f.write(json.dumps(r, ensure_ascii=False) + "\n")
    return {"train": len(rows) - nval, "val": nval}


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out-dir", required=True)
    ap.add_argument("--source", action="append", default=[], help="name=hub_id or local:<glob> (default: built-in)")
    ap.add_argument("--max-per-source", type=int, default=200_000)
    ap.add_argument("--min-chars", type=int, default=20)
    ap.add_argument("--max-chars", type=int, default=12_000)
    ap.add_argument("--val-frac", type=float, default=0.01)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    if args.source:
        sources = [Source(s.split("=", 1)[0] if "=" in s else s, s.split("=", 1)[-1]) for s in args.source]
    else:
        sources = DEFAULT_SOURCES
    rows, stats = collect(sources, args.max_per_source, args.min_chars, args.max_chars)
    print(json.dumps({"per_source": stats, **write_split(rows, Path(args.out_dir), args.val_frac, args.seed)}))


if __name__ == "__main__":
    main()
