"""Prune a byte-level BPE tokenizer to a smaller vocabulary chosen by frequency on a corpus.

A large multilingual vocabulary spends rows on scripts a model will not see.  This keeps
the tokens that occur most often on a representative corpus plus what keeps the
tokenizer *complete* and *consistent*:

* every byte-level base symbol (any string stays encodable);
* every special / added token;
* the merge closure of every kept token (each kept multi-symbol token is reachable
  through merges whose parts are kept), so encoding with the pruned merge list produces
  only kept tokens.

Outputs under ``--output``: ``tokenizer.json`` (the source pipeline with the pruned
vocab and merges, ids renumbered in source-id order), the tokenizer's config files,
``embedding_row_map.npy`` (``row_map[new_id] = old_id``, to initialise an embedding as
``old_embedding[row_map]``) and ``prune_report.json``.  Selection is by frequency, never
by id range: a CJK block may sit far from the low ids.  (Same outputs as the reference's
``scripts/prune_tokenizer.py``.)

    python -m myk_llm_b200.data.prune_tokenizer --source TOK --corpus data/corpus_en.txt data/corpus_zh.txt \\
        --vocab-size 65536 --output TOK-pruned64k
"""

from __future__ import annotations

import argparse
import json
import shutil
from collections import Counter
from pathlib import Path
from typing import Iterable

import numpy as np


def byte_symbols() -> list[str]:
    """The 256 base symbols of byte-level BPE (printable bytes map to themselves, the rest
    to code points from 256 upwards)."""
    printable = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    table, extra = {}, 0
    for b in range(256):
        if b in printable:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return [table[b] for b in range(256)]


def merge_pair(merge) -> tuple[str, str]:
    if isinstance(merge, (list, tuple)):
        return merge[0], merge[1]
    a, b = merge.split(" ", 1)
    return a, b


def closure(token: str, parents: dict[str, tuple[str, str]], memo: dict[str, frozenset]) -> frozenset:
    """The token plus every token its merges are built from."""
    if token in memo:
        return memo[token]
    out, stack = {token}, [token]
    while stack:
        t = stack.pop()
        if t in memo:
            out |= memo[t]
            continue
        for p in parents.get(t, ()):
            if p not in out:
                out.add(p)
                stack.append(p)
    memo[token] = frozenset(out)
    return memo[token]


def count_frequencies(tokenizer, lines: Iterable[str], vocab_size: int, batch: int = 1024) -> np.ndarray:
    counts = np.zeros(vocab_size, dtype=np.int64)
    buf: list[str] = []

    def flush():
        for enc in tokenizer.encode_batch(buf, add_special_tokens=False):
            np.add.at(counts, np.asarray(enc.ids, dtype=np.int64), 1)
        buf.clear()

    for line in lines:
        if line.strip():
            buf.append(line.rstrip("\n"))
            if len(buf) >= batch:
                flush()
    if buf:
        flush()
    return counts


def prune(tok_json: dict, counts: np.ndarray, target: int) -> tuple[dict, np.ndarray, dict]:
    model = tok_json["model"]
    if model.get("type") != "BPE":
        raise ValueError("only BPE tokenizers can be pruned")
    vocab: dict[str, int] = model["vocab"]
    merges = [merge_pair(m) for m in model["merges"]]
    parents = {a + b: (a, b) for a, b in merges}
    inv = {i: t for t, i in vocab.items()}
    keep = {s for s in byte_symbols() if s in vocab}
    specials = {a["content"] for a in tok_json.get("added_tokens", []) if a["content"] in vocab}
    keep |= specials
    memo: dict[str, frozenset] = {}
    for tid in np.argsort(-counts, kind="stable"):
        if counts[tid] == 0 or len(keep) >= target:
            break
        t = inv.get(int(tid))
        if t is None or t in keep:
            continue
        need = closure(t, parents, memo) - keep
        if len(keep) + len(need) <= target:
            keep |= need
    old_ids = sorted(vocab[t] for t in keep)
    new_vocab = {inv[o]: n for n, o in enumerate(old_ids)}
    new_merges = [f"{a} {b}" for a, b in merges if a in keep and b in keep and a + b in keep]
    out = json.loads(json.dumps(tok_json))
    out["model"]["vocab"] = new_vocab
    out["model"]["merges"] = new_merges
    for a in out.get("added_tokens", []):
        a["id"] = new_vocab[a["content"]] if a["content"] in new_vocab else a["id"]
    row_map = np.asarray(old_ids, dtype=np.int64)
    report = {"source_vocab": len(vocab), "kept": len(keep), "merges_kept": len(new_merges),
              "merges_source": len(merges), "specials": len(specials),
              "corpus_tokens": int(counts.sum()),
              "corpus_coverage_of_kept": float(counts[row_map].sum() / max(1, counts.sum()))}
    return out, row_map, report


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--source", required=True, help="tokenizer directory (tokenizer.json)")
    ap.add_argument("--corpus", nargs="+", required=True)
    ap.add_argument("--vocab-size", type=int, default=65536)
    ap.add_argument("--output", required=True)
    ap.add_argument("--max-lines", type=int, default=0)
    args = ap.parse_args(argv)
    from tokenizers import Tokenizer

    src = Path(args.source)
    tok = Tokenizer.from_file(str(src / "tokenizer.json"))

    def lines():
        n = 0
        for p in args.corpus:
            with open(p, encoding="utf-8") as f:
                for line in f:
                    yield line
                    n += 1
                    if args.max_lines and n >= args.max_lines:
                        return

    counts = count_frequencies(tok, lines(), tok.get_vocab_size(with_added_tokens=True))
    tj = json.loads((src / "tokenizer.json").read_text(encoding="utf-8"))
    new, row_map, report = prune(tj, counts, args.vocab_size)
    out = Path(args.output)
    out.mkdir(parents=True, exist_ok=True)
    (out / "tokenizer.json").write_text(json.dumps(new, ensure_ascii=False), encoding="utf-8")
    for extra in ("tokenizer_config.json", "special_tokens_map.json", "chat_template.jinja"):
        if (src / extra).exists():
            shutil.copy(src / extra, out / extra)
    np.save(out / "embedding_row_map.npy", row_map)
    (out / "prune_report.json").write_text(json.dumps(report, indent=2), encoding="utf-8")
    print(json.dumps(report))


if __name__ == "__main__":
    main()
