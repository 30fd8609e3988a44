"""Concatenate every file under a directory with one of the given extensions into one
text file, in random order (a quick corpus from a source tree, e.g. for tokenizer
frequency counts); prints the files it took.  The reference's ``scripts/aggregate.py``::

    python -m myk_llm_b200.utils.aggregate src/ .py,.md corpus_code.txt
"""

from __future__ import annotations

import argparse
import os
import random
import sys


def find_files(directory: str, extensions: list[str]) -> list[str]:
    out = []
    for root, _dirs, files in os.walk(directory):
        out.extend(os.path.join(root, f) for f in files if f.endswith(tuple(extensions)))
    return sorted(out)


def aggregate(directory: str, extensions: list[str], output: str, seed: int | None = None) -> list[str]:
    files = find_files(directory, extensions)
    random.Random(seed).shuffle(files)
    taken = []
    with open(output, "w", encoding="utf-8") as dst:
        for path in files:
            try:
                with open(path, encoding="utf-8") as src:
                    dst.write(src.read())
                taken.append(path)
            except (OSError, UnicodeDecodeError) as err:
                print(f"skipping {path}: {err}", file=sys.stderr)
    return taken


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("directory")
    ap.add_argument("extensions", help="comma-separated, e.g. .py,.txt")
    ap.add_argument("output")
    ap.add_argument("--seed", type=int, default=None)
    args = ap.parse_args(argv)
    taken = aggregate(args.directory, args.extensions.split(","), args.output, args.seed)
    print(f"Aggregated {len(taken)} files into {args.output}")
    for path in taken:
        print(path)


if __name__ == "__main__":
    main()
