"""How often a model's multi-token-prediction (MTP) drafts would be accepted by greedy
speculative decoding with K = 0 .. depth drafts per step (the quantity the speculative
decoders turn into speed).

At position ``i`` the main model's greedy token is ``g(i)`` and MTP head ``k`` drafts
``d_k(i)`` for position ``i + 1 + k``.  Draft ``k`` is accepted when ``d_j(i) = g(i + j)``
for every ``j <= k`` (a chain).  Per K the report gives the chained acceptance ``a_k``,
tokens per verify step ``E = 1 + a_1 + ... + a_K``, bytes per step, and the sampling
(T = 1) acceptance of the greedy drafts, ``prod_j p(d_j(i) | x_<=i+j)``.  As in the
reference's ``scripts/eval_mtp_acceptance.py``, two texts are measured: teacher-forced
validation text (``text``), and the model's own greedy continuation of validation prompts
(``greedy``, exact for greedy speculative decoding; ``repeat`` is the share of repeated
4-grams in it).

All depths are scored at once: drafts and greedy targets are (K, T) tensors, the chain is
a cumulative product along K and the T = 1 acceptance a cumulative sum of log-probs.

    python -m myk_llm_b200.infer.eval_mtp_acceptance runs/sweeps/ngram-mtp/v32k-none
"""

from __future__ import annotations

import argparse
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch
import yaml


def _ahead(x: torch.Tensor, k: int, fill) -> torch.Tensor:
    """``x`` shifted left by ``k`` along the last dim, padded with ``fill``."""
    out = torch.full_like(x, fill)
    if k < x.shape[-1]:
        out[..., :x.shape[-1] - k] = x[..., k:]
    return out


@torch.no_grad()
def row_acceptance(model, ids: torch.Tensor, targets: torch.Tensor, seqlens, token_bytes: torch.Tensor,
                   start: int = 0) -> dict[str, np.ndarray]:
    """One row (1, T): accepted[k, i] (chained), p_accepted[k, i], the bytes of each draft
    and of the verified token, over positions whose next ``depth + 1`` targets are all
    in-document (and at or after ``start``)."""
    from ..data.config import IGNORE_INDEX
    from ..train.objectives import mtp_targets

    out = model(ids, seqlens=seqlens)
    heads = model.mtp_hidden(out, ids)
    depth = len(heads)
    logp = model.logits(out.hidden[0]).float().log_softmax(-1)          # (T, V)
    greedy = logp.argmax(-1)                                              # (T,)
    drafts = torch.stack([model.logits(h[0]).float().argmax(-1) for h in heads])  # (K, T)
    wanted = torch.stack([_ahead(greedy, k, -1) for k in range(1, depth + 1)])
    chained = (drafts == wanted).long().cumprod(0).bool()
    # log p of draft k under the main model at the position it is verified (i + k)
    draft_lp = torch.stack([_verify_logp(logp, drafts[k - 1], k) for k in range(1, depth + 1)])
    p_chain = draft_lp.cumsum(0).exp()
    keep = mtp_targets(targets, depth)[0] != IGNORE_INDEX
    keep[:start] = False
    tb = token_bytes.to(ids.device)
    return {"accepted": chained[:, keep].float().cpu().numpy(), "p_accepted": p_chain[:, keep].cpu().numpy(),
            "bytes": tb[drafts][:, keep].cpu().numpy(), "first_bytes": tb[greedy][keep].cpu().numpy()}


def _verify_logp(logp: torch.Tensor, draft: torch.Tensor, k: int) -> torch.Tensor:
    """``log p(draft(i) | x_<=i+k)``: row ``i + k`` of the main model's log-probs at the
    draft's token; ``-inf`` where ``i + k`` is past the end."""
    t = logp.shape[0]
    out = torch.full((t,), float("-inf"), device=logp.device)
    if k < t:
        out[:t - k] = logp[k:].gather(1, draft[:t - k, None])[:, 0]
    return out


def summarize(parts: list[dict[str, np.ndarray]]) -> dict:
    """Per K in 0..depth: a_k, expected tokens / bytes per step, T = 1 acceptance."""
    cat = {key: np.concatenate([p[key] for p in parts], axis=-1) for key in parts[0]}
    acc, pacc, nbytes, first = cat["accepted"], cat["p_accepted"], cat["bytes"], cat["first_bytes"]
    run_tokens = np.concatenate([np.zeros((1, acc.shape[1])), np.cumsum(acc, 0)])
    run_bytes = np.concatenate([np.zeros((1, acc.shape[1])), np.cumsum(acc * nbytes, 0)])
    run_p = np.concatenate([np.zeros((1, acc.shape[1])), np.cumsum(pacc, 0)])
    rows = [{"K": k,
             "a_k": float(acc[k - 1].mean()) if k else 1.0,
             "tokens_per_iter": float((1 + run_tokens[k]).mean()),
             "bytes_per_iter": float((first + run_bytes[k]).mean()),
             "p_accept_k": float(pacc[k - 1].mean()) if k else 1.0,
             "p_tokens_per_iter": float((1 + run_p[k]).mean())} for k in range(acc.shape[0] + 1)]
    return {"positions": int(acc.shape[1]), "rows": rows}


def repeat_fraction(ids: list[int], n: int = 4) -> float:
    """Share of n-grams that already occurred earlier in the sequence."""
    grams = list(zip(*(ids[i:] for i in range(n))))
    first_seen = {}
    for pos, g in enumerate(grams):
        first_seen.setdefault(g, pos)
    repeats = sum(1 for pos, g in enumerate(grams) if first_seen[g] < pos)
    return repeats / max(1, len(grams))


def _report(name: str, text: dict, greedy: dict, reps: list[float]) -> None:
    print(f"\n{name}: text {text['positions']} positions; greedy {greedy['positions']} positions, "
          f"repeated 4-grams {100 * np.mean(reps):.0f}%")
    print("| K | text a_k | text tok/iter | text B/iter | p_accept_k (T=1) | greedy a_k | greedy tok/iter "
          "| greedy B/iter |")
    print("|---|---|---|---|---|---|---|---|")
    for t, g in zip(text["rows"], greedy["rows"]):
        print(f"| {t['K']} | {t['a_k']:.3f} | {t['tokens_per_iter']:.3f} | {t['bytes_per_iter']:.2f} | "
              f"{t['p_accept_k']:.3f} | {g['a_k']:.3f} | {g['tokens_per_iter']:.3f} | {g['bytes_per_iter']:.2f} |")


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
    from ..train.checkpoint import latest_checkpoint
    from ..train.config import TrainConfig
    from ..train.trainer import token_byte_lengths

    for run in map(Path, args.run_dirs):
        cfg = from_dict(TrainConfig, yaml.safe_load((run / "config.yaml").read_text()))
        ckpt = latest_checkpoint(run)
        if ckpt is None:
            print(f"{run.name}: no complete checkpoint")
            continue
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
                parts.append(row_acceptance(model, ids, tgt, [torch.tensor([ids.shape[1]], device="cuda")], tb,
                                            start=args.prompt_len))
                reps.append(repeat_fraction(ids[0, args.prompt_len:].tolist()))
            _report(val.name, text, summarize(parts), reps)


if __name__ == "__main__":
    main()
