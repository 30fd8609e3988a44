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
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

from ..configuration import load_config
from ..models import MykLLM
from ..utils.sweep import SEED_SUFFIX
from ..utils.testbed import autocast_for
from .eval import answer_positions
from .tasks import Example, make_example

SIGNALS = ("delta", "kl", "conf", "correct")
RULES = ([("delta", "<", t) for t in (0.2, 0.1, 0.05, 0.02, 0.01)]
         + [("kl", "<", t) for t in (0.1, 0.01, 1e-3, 1e-4)] + [("conf", ">", t) for t in (0.9, 0.99, 0.999)])
SHOWN = (2, 3, 4, 5, 6, 7, 8, 10, 12, 16, 24)


class _LoopReader:
    """Collects the final-normed loop state at the answer positions after every core
    iteration (through ``MykLLM.core_observer``)."""

    def __init__(self, model: MykLLM, rows: torch.Tensor, cols: torch.Tensor) -> None:
        self.model, self.rows, self.cols = model, rows, cols
        self.states: list[torch.Tensor] = []

    def __call__(self, iteration: int, state: torch.Tensor) -> None:
        self.states.append(self.model.final_norm(state[self.rows, self.cols]).float())


def _per_query(values: torch.Tensor, spans: list[tuple[int, int]], reduce) -> np.ndarray:
    """(queries, iterations) from (iterations, positions) by reducing each query's span."""
    return torch.stack([reduce(values[:, lo:hi], dim=1) for lo, hi in spans]).cpu().numpy()


@torch.no_grad()
def trace(model: MykLLM, examples: list[Example], iterations: int) -> dict[str, np.ndarray]:
    """{signal: (queries, iterations)} for examples of one length; ``delta`` and ``kl``
    are inf at the first iteration (nothing to compare with)."""
    loop = model.config.loop
    if not loop.core or loop.prelude + loop.core != len(model.layers):
        raise ValueError("needs a looped model whose core is its last blocks")
    dev = model.device
    ids = torch.as_tensor(np.stack([e.ids for e in examples]), device=dev)
    rows, cols, spans = answer_positions(examples, dev)
    reader = _LoopReader(model, rows, cols)
    model.core_observer = reader
    try:
        with autocast_for(dev):
            model(ids, seqlens=[torch.tensor([ids.shape[1]])] * ids.shape[0], iterations=iterations)
    finally:
        model.core_observer = None
    h = torch.stack(reader.states)                               # (iterations, positions, hidden)
    logp = model.logits(h).float().log_softmax(-1)
    first = torch.full_like(h[:1, :, 0], float("inf"))
    change = (h[1:] - h[:-1]).norm(dim=-1) / h[1:].norm(dim=-1)
    kl = (logp[1:].exp() * (logp[1:] - logp[:-1])).sum(-1)
    right = (logp.argmax(-1) == ids[rows, cols + 1]).float()
    return {"delta": _per_query(torch.cat([first, change]), spans, torch.amax),
            "kl": _per_query(torch.cat([first, kl]), spans, torch.amax),
            "conf": _per_query(logp.amax(-1).exp(), spans, torch.amin),
            "correct": _per_query(right, spans, torch.amin)}


def exit_iterations(signal: np.ndarray, op: str, threshold: float, budget: int) -> np.ndarray:
    """Per query, the first iteration t >= 2 (1-based) whose signal passes the threshold,
    else ``budget``."""
    window = signal[:, 1:budget]
    passed = np.less(window, threshold) if op == "<" else np.greater(window, threshold)
    first = np.argmax(passed, axis=1) + 2
    return np.where(passed.any(axis=1), first, budget)


def _load_run(run: Path, device: torch.device):
    from .train import LcConfig

    cfg = load_config(LcConfig, run / "config.yaml")
    model = MykLLM(cfg.model).to(device)
    model.load_state_dict(torch.load(run / "model.pt", map_location=device)["state_dict"])
    return cfg, model.eval()


def analyze(run: Path, length: int, examples: int, iterations: int, hops: list[int] | None, force: bool,
            device: str | None = None) -> dict:
    """Traces of one run (cached in ``<run>/halting.npz`` for the same settings)."""
    cache = run / "halting.npz"
    settings = np.array([length, examples, iterations, *(hops or [])])
    if cache.exists() and not force:
        saved = dict(np.load(cache))
        if np.array_equal(saved["settings"], settings):
            return saved
    cfg, model = _load_run(run, torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu")))
    task = replace(cfg.task, hops=hops or cfg.task.eval_hops or cfg.task.hops)
    rng = np.random.default_rng([12345, length])
    pool = [make_example(rng, task, length) for _ in range(examples)]
    step = max(1, 65536 // length)
    parts = [trace(model, pool[lo:lo + step], iterations) for lo in range(0, len(pool), step)]
    loop = cfg.model.loop
    out = {name: np.concatenate([p[name] for p in parts]) for name in SIGNALS}
    out["hops"] = np.array([h for e in pool for h in e.hops])
    out["settings"] = settings
    out["budget"] = np.array(loop.train_iterations[1] if loop.train_iterations else loop.iterations)
    np.savez(cache, **out)
    return out


def _md(header: list[str], rows: list[list[str]]) -> list[str]:
    return ["| " + " | ".join(header) + " |", "|" + "---|" * len(header)] + ["| " + " | ".join(r) + " |" for r in rows]


_VIEWS = (("correct", "accuracy (%)", np.mean, lambda v: f"{100 * v:.0f}"),
          ("delta", "median state change", np.median, lambda v: f"{v:.3f}"),
          ("kl", "median KL to the previous iteration", np.median, lambda v: f"{v:.0e}"))


def tables(name: str, data: dict, budget: int) -> list[str]:
    """Markdown: each signal by hop count and iteration, then every exit rule's accuracy
    and mean iterations."""
    hop = data["hops"]
    hop_values = sorted(set(hop.tolist()))
    shown = [t for t in SHOWN if t <= data["correct"].shape[1]]
    out = [f"\n### {name} ({len(hop)} queries, exit budget {budget})\n"]
    for signal, title, stat, fmt in _VIEWS:
        rows = [[str(h)] + [fmt(v) for v in stat(data[signal][hop == h], axis=0)[[t - 1 for t in shown]]]
                for h in hop_values]
        out += [f"\n{title} by hop count (rows) and iteration (columns)\n"] + _md(["hops", *map(str, shown)], rows)
    correct = data["correct"][:, :budget]
    solved = correct.max(axis=1) > 0
    rules = {f"fixed r = {budget}": np.full(len(correct), budget),
             "oracle (first correct iteration)": np.where(solved, correct.argmax(axis=1) + 1, budget)}
    for signal, op, threshold in RULES:
        rules[f"{signal} {op} {threshold:g}"] = exit_iterations(data[signal], op, threshold, budget)
    groups = [np.ones(len(hop), dtype=bool)] + [hop == h for h in hop_values]
    rows = []
    for label, stop in rules.items():
        right = data["correct"][np.arange(len(stop)), stop - 1]
        rows.append([label] + [f"{100 * right[g].mean():.0f} ({stop[g].mean():.1f})" for g in groups])
    out += ["\nExit rules: accuracy % (mean iterations) by hop count\n"]
    out += _md(["rule", "all", *map(str, hop_values)], rows)
    return out


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
    pooled: dict[str, list[dict]] = {}
    for run in map(Path, args.runs):
        key = f"{run.parent.name}/{SEED_SUFFIX.sub('', run.name)}"
        pooled.setdefault(key, []).append(analyze(run, args.length, args.examples, args.iterations, args.hops,
                                                  args.force))
    for name, runs in pooled.items():
        merged = {k: np.concatenate([r[k] for r in runs]) for k in (*SIGNALS, "hops")}
        print("\n".join(tables(f"{name}, {len(runs)} runs", merged, args.budget or int(runs[0]["budget"]))))


if __name__ == "__main__":
    main()
