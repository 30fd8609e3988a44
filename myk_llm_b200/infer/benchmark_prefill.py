"""Prefill time and inference-cache size of model variants (random weights, one GPU).

"prefill" is :func:`~myk_llm_b200.models.generate`'s first pass (``use_cache=True,
keep_last=1``: a decoder-decoder runs its cross-decoder on the last position only);
"full" is a training-style forward over every position without a cache.  The cache size
counts every tensor the cache holds (attention keys / values, DeltaNet states)::

    python -m myk_llm_b200.infer.benchmark_prefill configs/lc/base.yaml \\
        --variants model.layer_pattern=LLLLXXXX model.layer_pattern=LLLG --lengths 8192 65536
"""

from __future__ import annotations

import argparse
import json
from typing import Any

import torch


def tensor_bytes(entry: Any) -> int:
    if isinstance(entry, torch.Tensor):
        return entry.numel() * entry.element_size()
    if isinstance(entry, (list, tuple)):
        return sum(tensor_bytes(e) for e in entry)
    if isinstance(entry, dict):
        return sum(tensor_bytes(e) for e in entry.values())
    if hasattr(entry, "__dict__"):
        return sum(tensor_bytes(v) for v in vars(entry).values())
    return 0


def _time(fn) -> float:
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    out = fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1), out


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config")
    ap.add_argument("overrides", nargs="*")
    ap.add_argument("--variants", nargs="*", default=[""], help="comma-separated extra overrides per variant")
    ap.add_argument("--lengths", type=int, nargs="+", default=[4096])
    ap.add_argument("--batch", type=int, default=1)
    args = ap.parse_args(argv)
    from ..configuration import load_config
    from ..models import MykLLM
    from ..train.config import TrainConfig

    for var in args.variants:
        extra = [v for v in var.split(",") if v]
        cfg = load_config(TrainConfig, args.config, args.overrides + extra).model
        for L in args.lengths:
            cfg.max_seq_len = max(cfg.max_seq_len, L)
            torch.manual_seed(0)
            model = MykLLM(cfg).cuda().eval()
            ids = torch.randint(0, cfg.vocab_size, (args.batch, L), device="cuda")
            with torch.no_grad():
                t_pre, out = _time(lambda: model(ids, use_cache=True, keep_last=1))
                t_full, _ = _time(lambda: model(ids))
            print(json.dumps({"variant": var or "base", "length": L, "batch": args.batch, "prefill_ms": t_pre,
                              "full_ms": t_full, "cache_mb": tensor_bytes(out.cache) / 2**20,
                              "prefill_tokens_per_s": args.batch * L / t_pre * 1e3}), flush=True)
            del model
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
