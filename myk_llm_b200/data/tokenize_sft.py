"""Tokenize chat JSONL / JSON into the packed, loss-masked SFT format
(:mod:`myk_llm_b200.data.sft`: ``P.tokens.bin``, ``P.loss_mask.bin``, ``P.spans.npy``,
``P.meta.json``) with the tokenizer's chat template (``{% generation %}`` gives the mask)::

    python -m myk_llm_b200.data.tokenize_sft --data data/sft/train.jsonl --tokenizer TOK --output data/sft/train
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Any, Iterator

from .sft import write_chat_dataset


def read_examples(path: Path) -> Iterator[dict[str, Any]]:
    if path.suffix == ".jsonl":
        with path.open(encoding="utf-8") as f:
            for line in f:
                if line.strip():
                    yield json.loads(line)
    else:
        data = json.loads(path.read_text(encoding="utf-8"))
        yield from (data if isinstance(data, list) else data.get("data", []))


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--data", required=True)
    ap.add_argument("--tokenizer", required=True, help="tokenizer directory (AutoTokenizer) with a chat template")
    ap.add_argument("--chat-template", default=None, help="jinja file overriding the tokenizer's template")
    ap.add_argument("--output", required=True, help="output prefix")
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(args.tokenizer)
    if args.chat_template:
        tok.chat_template = Path(args.chat_template).read_text(encoding="utf-8")
    meta = write_chat_dataset(tok, read_examples(Path(args.data)), args.output, args.tokenizer)
    print(json.dumps(meta))


if __name__ == "__main__":
    main()
