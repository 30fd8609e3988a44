"""Draft acceptance of a model's multi-token-prediction (MTP) heads for greedy
speculative decoding with K = 0..depth drafts (the quantity ``MTPDecoder`` /
``StaticDecoder`` turn into speed).

At position i the main model's greedy token is g(i) and MTP depth k drafts d_k(i) (the
token at i + 1 + k).  Draft k is accepted when d_j(i) == g(i + j) for every j <= k (a
chain).  Per K it reports the chained acceptance a_k, tokens per verify iteration
E = 1 + a_1 + ... + a_K, bytes per iteration, and the sampling (T = 1) acceptance of the
greedy drafts, prod_j p(d_j(i) | x_<=i+j).  Two text sources, like the reference's
``scripts/eval_mtp_acceptance.py``:

* ``text``   teacher-forced validation text (a proxy: decoding conditions on the model's
  own continuation);
* ``greedy`` the model continues validation prompts greedily, then the same measurement
  runs on its own continuation (exact for greedy speculative decoding on that text;
  ``repeat`` is the share of repeated 4-grams, which small models produce a lot of).

    python -m myk_llm_b200.infer.eval_mtp_acceptance runs/sweeps/ngram-mtp/v32k-none
"""

from __future__ import annotations

import argparse
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch
import yaml


@torch.no_grad()
def row_acceptance(model, ids: torch.Tensor, targets: torch.Tensor, seqlens, token_bytes: torch.Tensor,
                   start: int = 0) -> dict[str, np.ndarray]:
    """For one row (1, T): accepted[k, i] (chained), p_accepted[k, i], bytes of each draft
    and of the verified token, over positions whose next depth + 1 targets are in-document."""
    from ..data.config import IGNORE_INDEX
    from ..train.objectives import mtp_targets

    depth = len(model.mtp)
    out = model(ids, seqlens=seqlens)
    heads = model.mtp_hidden(out, ids)
    logits = model.logits(out.hidden[0]).float()
    greedy = logits.argmax(-1)
    logp = logits.log_softmax(-1)
    T = greedy.numel()
    keep = mtp_targets(targets, depth)[0] != IGNORE_INDEX
    keep[:start] = False
    chain = torch.ones(T, dtype=torch.bool, device=ids.device)
    pchain = torch.ones(T, device=ids.device)
    acc, pacc, nbytes = [], [], []
    tb = token_bytes.to(ids.device)
    for k, h in enumerate(heads, start=1):
        draft = model.logits(h[0]).float().argmax(-1)
        want = torch.full_like(greedy, -1)
        want[:-k] = greedy[k:]
        chain = chain & (draft == want)
        lp = torch.full((T,), float("-inf"), device=ids.device)
        lp[:-k] = logp[k:].gather(1, draft[:-k, None])[:, 0]
        pchain = pchain * lp.exp()
        acc.append(chain[keep].float())
        pacc.append(pchain[keep])
        nbytes.append(tb[draft][keep])
    return {"accepted": torch.stack(acc).cpu().numpy(), "p_accepted": torch.stack(pacc).cpu().numpy(),
            "bytes": torch.stack(nbytes).cpu().numpy(), "first_bytes": tb[greedy][keep].cpu().numpy()}


def summarize(parts: list[dict[str, np.ndarray]]) -> dict:
    """Per K in 0..depth: a_k, expected tokens / bytes per iteration, T = 1 acceptance."""
    cat = {key: np.concatenate([p[key] for p in parts], axis=-1) for key in parts[0]}
    a, p, b = cat["accepted"], cat["p_accepted"], cat["bytes"]
    rows = []
    for K in range(a.shape[0] + 1):
        rows.append({"K": K,
                     "a_k": float(a[K - 1].mean()) if K else 1.0,
                     "tokens_per_iter": float((1 + a[:K].sum(0)).mean()),
                     "bytes_per_iter": float((cat["first_bytes"] + (a[:K] * b[:K]).sum(0)).mean()),
                     "p_accept_k": float(p[K - 1].mean()) if K else 1.0,
                     "p_tokens_per_iter": float((1 + p[:K].sum(0)).mean())})
    return {"positions": int(a.shape[1]), "rows": rows}


def repeat_fraction(ids: list[int], n: int = 4) -> float:
    """Share of n-grams that already occurred earlier in the sequence."""
    grams = [tuple(ids[i:i + n]) for i in range(len(ids) - n + 1)]
    seen, rep = set(), 0
    for g in grams:
        rep += g in seen
        seen.add(g)
    return rep / max(1, len(grams))


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("run_dirs", nargs="+")
    ap.add_argument("--rows", type=int, default=64, help="validation rows per set")
    ap.add_argument("--prompts", type=int, default=64, help="greedy continuations per set")
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--new", type=int, default=256)
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    from ..configuration import from_dict
    from ..data import IGNORE_INDEX, build_fixed_batches
    from ..models import generate, load_model
    from ..train.config import TrainConfig
    from ..train.trainer import token_byte_lengths

    for run in map(Path, args.run_dirs):
        cfg = from_dict(TrainConfig, yaml.safe_load((run / "config.yaml").read_text()))
        ckpt = sorted((run / "checkpoints").glob("step_*"))[-1]
        model = load_model(ckpt)
        if not len(model.mtp):
            print(f"{run.name}: no MTP heads")
            continue
        tb = token_byte_lengths(AutoTokenizer.from_pretrained(cfg.data.tokenizer)).float()
        print(f"\n## {run.name} ({ckpt.name}, vocab {model.config.vocab_size}, MTP depth {len(model.mtp)})")
        for val in cfg.eval.val_sets:
            data = replace(cfg.data, sources=val.sources, micro_batch_size=1, kind=val.kind or cfg.data.kind)
            batches = build_fixed_batches(data, args.rows, cfg.eval.seed)
            text = summarize([row_acceptance(model, b.input_ids.cuda(), b.targets.cuda(),
                                             [s.cuda() for s in b.seqlens] if b.seqlens else None, tb)
                              for b in batches])
            parts, reps = [], []
            for b in batches[:args.prompts]:
                ids = generate(model, b.input_ids[:, :args.prompt_len].cuda(), args.new, temperature=0.0)
                tgt = torch.cat([ids[:, 1:], torch.full_like(ids[:, :1], IGNORE_INDEX)], 1)
                parts.append(row_acceptance(model, ids, tgt, [torch.tensor([ids.size(1)], device="cuda")], tb,
                                            start=args.prompt_len))
                reps.append(repeat_fraction(ids[0, args.prompt_len:].tolist()))
            greedy = summarize(parts)
            print(f"\n{val.name}: text {text['positions']} positions; greedy {greedy['positions']} positions, "
                  f"repeated 4-grams {100 * np.mean(reps):.0f}%")
            print("| K | text a_k | text tok/iter | text B/iter | p_accept_k (T=1) | greedy a_k | greedy tok/iter "
                  "| greedy B/iter |")
            print("|---|---|---|---|---|---|---|---|")
            for t, g in zip(text["rows"], greedy["rows"]):
                print(f"| {t['K']} | {t['a_k']:.3f} | {t['tokens_per_iter']:.3f} | {t['bytes_per_iter']:.2f} | "
                      f"{t['p_accept_k']:.3f} | {g['a_k']:.3f} | {g['tokens_per_iter']:.3f} | "
                      f"{g['bytes_per_iter']:.2f} |")


if __name__ == "__main__":
    main()
