"""Tokenize a text corpus into token shards (:mod:`myk_llm_b200.data.shards`).

The corpus is streamed (a HuggingFace dataset id or local json/jsonl/parquet/text files),
documents pass the same :class:`~myk_llm_b200.data.filters.DocFilter` as streaming
training, and ``<output>/train`` and ``<output>/val`` receive shard sets.  ``--workers N``
runs N processes, each reading a disjoint 1/N of the stream into its own shard prefix
(behaviour of the reference's ``scripts/pretokenize.py:37-126``)::

    python -m myk_llm_b200.data.pretokenize --hf-path HuggingFaceFW/fineweb-edu --hf-config sample-10BT \\
        --tokenizer _download_models/Qwen3.5-0.8B-pruned64k --target-tokens 5e9 --output data/shards/en --workers 8
    python -m myk_llm_b200.data.pretokenize --path 'corpus/*.jsonl' --tokenizer tok --target-tokens 1e8 --output out
"""

from __future__ import annotations

import argparse
import json
import multiprocessing as mp
from pathlib import Path

from .config import SourceConfig
from .filters import DocFilter
from .shards import ShardWriter, write_meta_file
from .streaming import open_stream


def _load_tokenizer(path: str):
    from tokenizers import Tokenizer

    return Tokenizer.from_file(str(Path(path) / "tokenizer.json"))


def run_worker(args, worker: int, workers: int, tokenizer=None, open_fn=open_stream) -> dict:
    """One worker: its share of the stream -> train / val shards until its token budget."""
    tok = tokenizer if tokenizer is not None else _load_tokenizer(args.tokenizer)
    eos = args.eos_id if args.eos_id is not None else tok.token_to_id(args.eos_token)
    if eos is None:
        raise ValueError(f"{args.eos_token!r} is not in the tokenizer vocabulary")
    src = SourceConfig(name="corpus", path=args.path or "", hf_path=args.hf_path or "", hf_config=args.hf_config,
                       hf_split=args.hf_split, text_key=args.text_key)
    stream = open_fn(src, args.seed, args.shuffle_buffer, worker, workers)
    flt = DocFilter(max_doc_tokens=args.max_doc_tokens)
    out = Path(args.output)
    prefix = f"w{worker:03d}"
    train = ShardWriter(out / "train", eos, args.tokenizer or "", shard_tokens=int(float(args.shard_tokens)),
                        prefix=prefix)
    val = ShardWriter(out / "val", eos, args.tokenizer or "", shard_tokens=int(float(args.shard_tokens)), prefix=prefix)
    budget = int(float(args.target_tokens)) // workers
    kept = dropped = 0
    batch: list[str] = []

    def flush() -> None:
        nonlocal kept, dropped
        for enc in tok.encode_batch(batch, add_special_tokens=False):
            ids = list(enc.ids)
            if flt.max_doc_tokens and len(ids) > flt.max_doc_tokens:
                ids = ids[:flt.max_doc_tokens]
            if not ids or flt.reject(ids):
                dropped += 1
                continue
            total = train.num_tokens + val.num_tokens + len(ids)
            (val if val.num_tokens < args.val_fraction * total else train).add(ids)
            kept += 1
        batch.clear()

    for ex in stream:
        text = ex.get(args.text_key)
        if not isinstance(text, str) or not text.strip() or flt.reject_text(text, args.script):
            dropped += 1
            continue
        batch.append(text)
        if len(batch) >= 256:
            flush()
            if train.num_tokens + val.num_tokens >= budget:
                break
    if batch:
        flush()
    n_train, n_val = train.num_tokens, val.num_tokens
    return {"worker": worker, "train_tokens": n_train, "val_tokens": n_val, "kept": kept, "dropped": dropped,
            "eos_id": eos, "train_shards": train.close(write_meta=False), "val_shards": val.close(write_meta=False)}


def _entry(a):
    args, w, n = a
    return run_worker(args, w, n)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--hf-path")
    src.add_argument("--path", help="local files (glob)")
    ap.add_argument("--hf-config", default=None)
    ap.add_argument("--hf-split", default="train")
    ap.add_argument("--text-key", default="text")
    ap.add_argument("--script", choices=["latin", "cjk"], default=None)
    ap.add_argument("--tokenizer", required=True, help="directory with tokenizer.json")
    ap.add_argument("--eos-token", default="<|endoftext|>")
    ap.add_argument("--eos-id", type=int, default=None)
    ap.add_argument("--target-tokens", default="1e9")
    ap.add_argument("--val-fraction", type=float, default=0.001)
    ap.add_argument("--shard-tokens", default=str(1 << 28))
    ap.add_argument("--max-doc-tokens", type=int, default=0)
    ap.add_argument("--shuffle-buffer", type=int, default=10_000)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workers", type=int, default=1)
    ap.add_argument("--output", required=True)
    args = ap.parse_args(argv)
    if args.workers == 1:
        stats = [run_worker(args, 0, 1)]
    else:
        with mp.get_context("spawn").Pool(args.workers) as pool:
            stats = pool.map(_entry, [(args, w, args.workers) for w in range(args.workers)])
    out = Path(args.output)
    for split in ("train", "val"):
        shards = [sh for s in stats for sh in s[f"{split}_shards"]]
        write_meta_file(out / split, shards, stats[0]["eos_id"], args.tokenizer, {"workers": args.workers})
    print(json.dumps({"train_tokens": sum(s["train_tokens"] for s in stats),
                      "val_tokens": sum(s["val_tokens"] for s in stats),
                      "kept": sum(s["kept"] for s in stats), "dropped": sum(s["dropped"] for s in stats)}))


if __name__ == "__main__":
    main()
