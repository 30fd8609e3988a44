"""Stream a token-budgeted raw-text sample of a corpus (e.g. the English + Chinese mix that
drives :mod:`myk_llm_b200.data.prune_tokenizer`): documents are tokenized only to count
real tokens, and text is written until the budget is reached::

    python -m myk_llm_b200.data.download_corpus --lang en --tokenizer TOK --target-tokens 50e6 --output data/corpus_en.txt
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

from .config import SourceConfig
from .streaming import open_stream

PRESETS = {"en": ("HuggingFaceFW/fineweb-edu", "sample-10BT"), "zh": ("opencsg/chinese-fineweb-edu-v2", None)}


def write_sample(stream, tokenizer, target_tokens: int, output: Path, text_key: str = "text") -> dict:
    n_tok = n_doc = 0
    output.parent.mkdir(parents=True, exist_ok=True)
    with output.open("w", encoding="utf-8") as f:
        for ex in stream:
            text = ex.get(text_key)
            if not isinstance(text, str) or not text.strip():
                continue
            n_tok += len(tokenizer.encode(text, add_special_tokens=False).ids)
            f.write(text.replace("\n", " ").strip() + "\n")
            n_doc += 1
            if n_tok >= target_tokens:
                break
    return {"tokens": n_tok, "documents": n_doc, "output": str(output)}


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--lang", choices=sorted(PRESETS), default=None)
    ap.add_argument("--hf-path", default=None)
    ap.add_argument("--hf-config", default=None)
    ap.add_argument("--path", default=None, help="local files instead of a hub dataset")
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--target-tokens", default="5e7")
    ap.add_argument("--output", required=True)
    args = ap.parse_args(argv)
    from tokenizers import Tokenizer

    hf_path, hf_config = PRESETS[args.lang] if args.lang else (args.hf_path or "", args.hf_config)
    src = SourceConfig(name="corpus", path=args.path or "", hf_path=hf_path, hf_config=hf_config)
    tok = Tokenizer.from_file(str(Path(args.tokenizer) / "tokenizer.json"))
    print(json.dumps(write_sample(open_stream(src, 0, 10_000), tok, int(float(args.target_tokens)), Path(args.output))))


if __name__ == "__main__":
    main()
