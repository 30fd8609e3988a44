"""Early-exit analysis of looped retrieval models: does the loop state settle once a
query's chain is resolved, so that a convergence signal could stop iterating?

    python -m myk_llm_b200.lc.halting runs/lc/loop/chain-h6-s{0,1,2} [--hops 1 2 ...]

Each checkpoint runs once at ``--iterations`` core iterations and is read out after
every iteration (the core must be the model's last blocks: the readout is the final
norm and the LM head applied to the loop state).  Per query, over the positions that
predict its answer:

* ``delta``: ||h_t - h_{t-1}|| / ||h_t|| of the final-normed state (max over positions)
* ``kl``: KL(p_t || p_{t-1}) of the next-token distributions (max)
* ``conf``: probability of the argmax token (min)
* ``correct``: exact match of the answer read at iteration t (min)

An exit rule stops a query at the first iteration t >= 2 whose signal passes a
threshold, else at the budget, and is scored by accuracy and mean iterations.  Traces go
to ``<run>/halting.npz`` (reused unless ``--force``); runs of one configuration (seed
suffix ``-s<k>``) are pooled.  (The reference's ``src/myk_llm/lc/halting.py:49-169``
defines the same signals and rules.)
"""

from __future__ import annotations

import argparse
import contextlib
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

from ..configuration import load_config
from ..models import MykLLM
from ..models.transformer import materialize
from ..utils.sweep import SEED_SUFFIX
from .eval import answer_positions
from .tasks import Example, make_example

SIGNALS = ("delta", "kl", "conf", "correct")
RULES = ([("delta", "<", t) for t in (0.2, 0.1, 0.05, 0.02, 0.01)]
         + [("kl", "<", t) for t in (0.1, 0.01, 1e-3, 1e-4)] + [("conf", ">", t) for t in (0.9, 0.99, 0.999)])
SHOWN = (2, 3, 4, 5, 6, 7, 8, 10, 12, 16, 24)


@torch.no_grad()
def trace(model: MykLLM, examples: list[Example], iterations: int) -> dict[str, np.ndarray]:
    """{signal: (queries, iterations)} for equal-length examples (delta / kl are inf at
    the first iteration)."""
    loop = model.config.loop
    if not loop.core or loop.prelude + loop.core != len(model.layers):
        raise ValueError("needs a looped model whose core is its last blocks")
    dev = model.device
    ids = torch.from_numpy(np.stack([e.ids for e in examples])).to(dev)
    rows, pos, spans = answer_positions(examples, dev)
    reads: list[torch.Tensor] = []

    def hook(_m, _a, out):
        x = materialize(out[0] if isinstance(out, tuple) else out)
        reads.append(model.final_norm(x[rows, pos]).float())

    handle = model.layers[-1].register_forward_hook(hook)
    amp = torch.autocast("cuda", dtype=torch.bfloat16) if dev.type == "cuda" else contextlib.nullcontext()
    try:
        with amp:
            model(ids, seqlens=[torch.tensor([ids.size(1)])] * ids.size(0), iterations=iterations)
    finally:
        handle.remove()
    h = torch.stack(reads)  # (iterations, positions, hidden)
    logp = torch.log_softmax(model.logits(h).float(), dim=-1)
    inf = torch.full_like(h[:1, :, 0], float("inf"))
    per = {"delta": torch.cat([inf, (h[1:] - h[:-1]).norm(dim=-1) / h[1:].norm(dim=-1)]),
           "kl": torch.cat([inf, (logp[1:].exp() * (logp[1:] - logp[:-1])).sum(-1)]),
           "conf": logp.max(-1).values.exp(),
           "correct": (logp.argmax(-1) == ids[rows, pos + 1]).float()}
    out = {}
    for name, v in per.items():
        red = torch.amin if name in ("conf", "correct") else torch.amax
        out[name] = torch.stack([red(v[:, a:b], dim=1) for a, b in spans]).cpu().numpy()
    return out


def exit_iterations(signal: np.ndarray, op: str, threshold: float, budget: int) -> np.ndarray:
    """First iteration (1-based, >= 2) whose signal passes, else ``budget``."""
    win = signal[:, 1:budget]
    ok = win < threshold if op == "<" else win > threshold
    return np.where(ok.any(1), ok.argmax(1) + 2, budget)


def analyze(run: Path, length: int, examples: int, iterations: int, hops: list[int] | None, force: bool,
            device: str | None = None) -> dict:
    from .train import LcConfig

    cache = run / "halting.npz"
    settings = np.array([length, examples, iterations, *(hops or [])])
    if cache.exists() and not force:
        st = np.load(cache)
        if np.array_equal(st["settings"], settings):
            return dict(st)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    cfg = load_config(LcConfig, run / "config.yaml")
    model = MykLLM(cfg.model).to(dev)
    model.load_state_dict(torch.load(run / "model.pt", map_location=dev)["state_dict"])
    model.eval()
    task = replace(cfg.task, hops=hops or cfg.task.eval_hops or cfg.task.hops)
    rng = np.random.default_rng([12345, length])
    pool = [make_example(rng, task, length) for _ in range(examples)]
    per = max(1, 65536 // length)
    parts = [trace(model, pool[i:i + per], iterations) for i in range(0, len(pool), per)]
    loop = cfg.model.loop
    res = {k: np.concatenate([p[k] for p in parts]) for k in SIGNALS}
    res |= {"hops": np.array([h for e in pool for h in e.hops]), "settings": settings,
            "budget": np.array(loop.train_iterations[1] if loop.train_iterations else loop.iterations)}
    np.savez(cache, **res)
    return res


def tables(name: str, data: dict, budget: int) -> list[str]:
    hops = sorted(set(data["hops"].tolist()))
    shown = [t for t in SHOWN if t <= data["correct"].shape[1]]
    lines = [f"\n### {name} ({len(data['hops'])} queries, exit budget {budget})\n"]
    for sig, title, fmt in (("correct", "accuracy (%)", lambda v: f"{100 * v:.0f}"),
                            ("delta", "median state change", lambda v: f"{v:.3f}"),
                            ("kl", "median KL to the previous iteration", lambda v: f"{v:.0e}")):
        lines += [f"\n{title} by hop count (rows) and iteration (columns)\n",
                  "| hops | " + " | ".join(map(str, shown)) + " |", "|---|" + "---|" * len(shown)]
        for h in hops:
            v = data[sig][data["hops"] == h]
            stat = v.mean(0) if sig == "correct" else np.median(v, 0)
            lines.append(f"| {h} | " + " | ".join(fmt(stat[t - 1]) for t in shown) + " |")
    corr = data["correct"]
    ever = corr[:, :budget].max(1) > 0
    rules = [(f"fixed r = {budget}", np.full(len(corr), budget)),
             ("oracle (first correct iteration)", np.where(ever, corr[:, :budget].argmax(1) + 1, budget))]
    rules += [(f"{s} {op} {t:g}", exit_iterations(data[s], op, t, budget)) for s, op, t in RULES]
    lines += ["\nExit rules: accuracy % (mean iterations) by hop count\n",
              "| rule | all | " + " | ".join(map(str, hops)) + " |", "|---|---|" + "---|" * len(hops)]
    for label, ex in rules:
        hit = corr[np.arange(len(ex)), ex - 1]
        masks = [slice(None)] + [data["hops"] == h for h in hops]
        lines.append(f"| {label} | " + " | ".join(f"{100 * hit[m].mean():.0f} ({ex[m].mean():.1f})" for m in masks)
                     + " |")
    return lines


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("runs", nargs="+")
    ap.add_argument("--length", type=int, default=2048)
    ap.add_argument("--examples", type=int, default=500)
    ap.add_argument("--iterations", type=int, default=24)
    ap.add_argument("--budget", type=int, default=None)
    ap.add_argument("--hops", type=int, nargs="*", default=None)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    groups: dict[str, list[dict]] = {}
    for run in map(Path, args.runs):
        d = analyze(run, args.length, args.examples, args.iterations, args.hops, args.force)
        groups.setdefault(f"{run.parent.name}/{SEED_SUFFIX.sub('', run.name)}", []).append(d)
    for name, runs in groups.items():
        pooled = {k: np.concatenate([r[k] for r in runs]) for k in (*SIGNALS, "hops")}
        print("\n".join(tables(f"{name}, {len(runs)} runs", pooled, args.budget or int(runs[0]["budget"]))))


if __name__ == "__main__":
    main()
