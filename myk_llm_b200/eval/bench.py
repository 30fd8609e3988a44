"""Zero-shot log-likelihood benchmarks for exported models and HuggingFace models.

Tasks and scoring follow EleutherAI lm-evaluation-harness conventions, as the reference's
``src/myk_llm/eval/bench.py:42-339`` does, so numbers are comparable across models:

* multiple choice (hellaswag, arc_easy / arc_challenge, piqa, xstorycloze_en/zh,
  xcopa_zh): the continuation with the highest total log-prob (``acc``) or the highest
  log-prob per character (``acc_norm``);
* winogrande: partial scoring (each option substituted into the blank, the shared
  remainder scored);
* lambada_openai: greedy last-word accuracy and last-word perplexity;
* bits per UTF-8 byte on raw documents (``bpb_*``): the first window scored from a
  newline, later chunks of window/2 tokens conditioned on the preceding window/2.

Scoring here packs many (context, continuation) requests into one varlen row set
(document-masked attention, no padding) and runs the LM head only on the continuation
positions, instead of padding a dense batch and materialising full-vocabulary logits.

    python -m myk_llm_b200.eval.bench --model runs/200m/export --tasks hellaswag,arc_easy --limit 500
    python -m myk_llm_b200.eval.bench --hf-model HuggingFaceTB/SmolLM2-135M --tasks piqa

Task data comes from ``datasets`` (hub ids, or ``--data-dir`` with local copies saved
under the task names).  Results are appended as one JSON line per model to ``--output``.
"""

from __future__ import annotations

import argparse
import json
import math
import re
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Iterable

import torch
import torch.nn.functional as F


# ------------------------------------------------------------------------------ models
class LogLikelihoodModel:
    """Scores (context, continuation) pairs.  Subclasses provide ``continuation_logprobs``."""

    name = "model"
    max_len = 2048
    tokenizer = None
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    num_params = 0

    def encode(self, text: str) -> list[int]:
        return list(self.tokenizer.encode(text, add_special_tokens=False))

    def loglikelihood(self, requests: list[tuple[str, str]]) -> list[tuple[float, bool, int]]:
        """Context and continuation tokenized separately and concatenated (lm-eval)."""
        enc = []
        for ctx, cont in requests:
            c = self.encode(cont)
            if not c:
                raise ValueError(f"empty continuation for context {ctx[:60]!r}")
            enc.append((self.encode(ctx), c))
        return self.loglikelihood_tokens(enc)

    @torch.no_grad()
    def loglikelihood_tokens(self, encoded: list[tuple[list[int], list[int]]],
                             tokens_per_batch: int = 32768) -> list[tuple[float, bool, int]]:
        """(sum log p(continuation | context), continuation is greedy, #continuation tokens)."""
        items = []
        for ctx, cont in encoded:
            full = (ctx + cont)[-(self.max_len + 1):]
            inputs = full[:-1]
            n = min(len(cont), len(inputs))
            items.append((inputs, full[-n:], len(inputs) - n))
        order = sorted(range(len(items)), key=lambda i: -len(items[i][0]))
        results: list[tuple[float, bool, int] | None] = [None] * len(items)
        i = 0
        while i < len(order):
            group, used = [], 0
            while i < len(order) and (not group or used + len(items[order[i]][0]) <= tokens_per_batch):
                group.append(order[i])
                used += len(items[order[i]][0])
                i += 1
            rows = [items[j] for j in group]
            for j, res in zip(group, self.continuation_logprobs(rows)):
                results[j] = res
        return results  # type: ignore[return-value]

    def continuation_logprobs(self, rows: list[tuple[list[int], list[int], int]]) -> list[tuple[float, bool, int]]:
        raise NotImplementedError


def _score(logits: torch.Tensor, targets: torch.Tensor) -> tuple[float, bool]:
    lp = F.log_softmax(logits.float(), dim=-1)
    return float(lp.gather(1, targets[:, None]).sum()), bool((logits.argmax(-1) == targets).all())


class MykModel(LogLikelihoodModel):
    """An exported model directory; requests are packed as documents of one varlen row."""

    def __init__(self, model_dir: str, max_len: int = 2048, device: str | None = None) -> None:
        from transformers import AutoTokenizer

        from ..models.io import load_model

        if device is not None:
            self.device = torch.device(device)
        self.model = load_model(model_dir, device=self.device).eval()
        self.tokenizer = AutoTokenizer.from_pretrained(model_dir)
        self.max_len = min(max_len, self.model.config.max_seq_len)
        self.name = "/".join(Path(model_dir).resolve().parts[-3:])
        self.num_params = self.model.num_parameters()

    def continuation_logprobs(self, rows):
        ids = torch.tensor([t for r in rows for t in r[0]], dtype=torch.long, device=self.device)[None]
        lens = torch.tensor([len(r[0]) for r in rows], dtype=torch.int32)
        ctx = torch.autocast("cuda", dtype=torch.bfloat16) if self.device.type == "cuda" else _null()
        with ctx:
            hidden = self.model(ids, seqlens=[lens]).hidden[0]
        out, base = [], 0
        for inputs, cont, lo in rows:
            h = hidden[base + lo: base + len(inputs)]
            logits = self.model.logits(h)
            tot, greedy = _score(logits, torch.tensor(cont, device=self.device))
            out.append((tot, greedy, len(cont)))
            base += len(inputs)
        return out


class HFModel(LogLikelihoodModel):
    """A HuggingFace causal LM (right-padded dense batches)."""

    def __init__(self, path: str, max_len: int = 2048) -> None:
        from transformers import AutoModelForCausalLM, AutoTokenizer

        self.tokenizer = AutoTokenizer.from_pretrained(path)
        self.model = AutoModelForCausalLM.from_pretrained(path, dtype=torch.bfloat16).to(self.device).eval()
        self.max_len = max_len
        self.name = path.rstrip("/").split("/")[-1]
        self.num_params = sum(p.numel() for p in self.model.parameters())

    def continuation_logprobs(self, rows):
        width = max(len(r[0]) for r in rows)
        ids = torch.zeros(len(rows), width, dtype=torch.long)
        for k, r in enumerate(rows):
            ids[k, :len(r[0])] = torch.tensor(r[0])
        logits = self.model(input_ids=ids.to(self.device)).logits
        return [(*_score(logits[k, lo:len(inp)], torch.tensor(cont, device=self.device)), len(cont))
                for k, (inp, cont, lo) in enumerate(rows)]


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ------------------------------------------------------------------------------- tasks
@dataclass
class MCExample:
    context: str
    choices: list[str]  # continuations, with any leading space
    label: int


def score_multiple_choice(model: LogLikelihoodModel, examples: list[MCExample]) -> dict[str, float]:
    reqs = [(e.context, c) for e in examples for c in e.choices]
    scores = model.loglikelihood(reqs)
    acc = acc_norm = k = 0
    for e in examples:
        lls = [s[0] for s in scores[k:k + len(e.choices)]]
        k += len(e.choices)
        norm = [ll / max(1, len(c)) for ll, c in zip(lls, e.choices)]
        acc += int(max(range(len(lls)), key=lls.__getitem__) == e.label)
        acc_norm += int(max(range(len(norm)), key=norm.__getitem__) == e.label)
    n = max(1, len(examples))
    return {"acc": acc / n, "acc_norm": acc_norm / n, "n": len(examples)}


DATA_DIR: Path | None = None


def _load(hub_id: str, *args, split: str, **kw):
    from datasets import load_dataset, load_from_disk

    if DATA_DIR is not None:
        local = DATA_DIR / (hub_id.replace("/", "__") + ("__" + args[0] if args else "") + f"__{split}")
        if local.exists():
            return load_from_disk(str(local))
    return load_dataset(hub_id, *args, split=split, **kw)


def _hs_clean(text: str) -> str:
    text = re.sub(r"\[.*?\]", "", text.strip().replace(" [title]", ". "))
    return text.replace("  ", " ")


def task_hellaswag(limit):
    out = []
    for r in _load("Rowan/hellaswag", split="validation"):
        ctx = _hs_clean(r["activity_label"] + ": " + r["ctx_a"] + " " + r["ctx_b"].capitalize())
        out.append(MCExample(ctx, [" " + _hs_clean(e) for e in r["endings"]], int(r["label"])))
    return out[:limit]


def task_arc(subset, limit):
    out = []
    for r in _load("allenai/ai2_arc", subset, split="test"):
        labels = r["choices"]["label"]
        if r["answerKey"] in labels:
            out.append(MCExample(f"Question: {r['question']}\nAnswer:", [" " + t for t in r["choices"]["text"]],
                                 labels.index(r["answerKey"])))
    return out[:limit]


def task_piqa(limit):
    rows = _load("ybisk/piqa", split="validation", revision="refs/convert/parquet")
    return [MCExample(f"Question: {r['goal']}\nAnswer:", [" " + r["sol1"], " " + r["sol2"]], int(r["label"]))
            for r in rows][:limit]


def task_xstorycloze(lang, limit):
    sep = "" if lang == "zh" else " "
    out = []
    for r in _load("juletxara/xstory_cloze", lang, split="eval"):
        ctx = sep.join(r[f"input_sentence_{i}"].strip() for i in range(1, 5))
        out.append(MCExample(ctx, [sep + r["sentence_quiz1"].strip(), sep + r["sentence_quiz2"].strip()],
                             int(r["answer_right_ending"]) - 1))
    return out[:limit]


def task_xcopa_zh(limit):
    out = []
    for r in _load("cambridgeltl/xcopa", "zh", split="test"):
        conn = "因为" if r["question"] == "cause" else "所以"
        out.append(MCExample(r["premise"].strip().rstrip("。.") + "，" + conn, [r["choice1"], r["choice2"]],
                             int(r["label"])))
    return out[:limit]


def winogrande_requests(rows) -> list[tuple[str, str]]:
    reqs = []
    for r in rows:
        b = r["sentence"].index("_")
        rest = " " + r["sentence"][b + 1:].strip()
        for opt in (r["option1"], r["option2"]):
            reqs.append((r["sentence"][:b] + opt, rest))
    return reqs


def eval_winogrande(model, limit, rows=None):
    rows = list(rows if rows is not None else _load("allenai/winogrande", "winogrande_xl", split="validation"))[:limit]
    s = model.loglikelihood(winogrande_requests(rows))
    ok = sum(int((0 if s[2 * i][0] > s[2 * i + 1][0] else 1) == int(r["answer"]) - 1) for i, r in enumerate(rows))
    return {"acc": ok / max(1, len(rows)), "n": len(rows)}


def eval_lambada(model, limit, rows=None):
    rows = list(rows if rows is not None else _load("EleutherAI/lambada_openai", "en", split="test"))[:limit]
    reqs = []
    for r in rows:
        ctx, word = r["text"].rsplit(" ", 1)
        reqs.append((ctx, " " + word))
    s = model.loglikelihood(reqs)
    return {"acc": sum(int(x[1]) for x in s) / max(1, len(rows)),
            "ppl": math.exp(-sum(x[0] for x in s) / max(1, len(rows))), "n": len(rows)}


def bpb_documents(name: str, limit: int | None) -> list[str]:
    n = limit or 300
    if name == "wikitext2":
        text = "".join(_load("Salesforce/wikitext", "wikitext-2-raw-v1", split="test")["text"])
        docs = [d for d in re.split(r"\n(?= = [^=].* = \n)", text) if d.strip()]
    elif name == "fineweb_edu_en":
        rows = _load("HuggingFaceFW/fineweb-edu", "sample-10BT", split="train", streaming=True)
        docs = [r["text"] for r in rows.skip(200_000).take(n)]
    elif name == "fineweb_edu_zh":
        rows = _load("opencsg/Fineweb-Edu-Chinese-V2.1", split="train", streaming=True, data_dir="4_5")
        docs = [r["text"] for r in rows.skip(200_000).take(n)]
    elif name == "wiki_zh":
        rows = _load("wikimedia/wikipedia", "20231101.zh", split="train", streaming=True)
        docs = [r["text"] for r in rows.skip(50_000).take(4 * n) if len(r["text"]) > 400]
    else:
        raise ValueError(f"unknown bpb corpus {name!r}")
    return docs[:n]


def eval_bpb(model: LogLikelihoodModel, docs: list[str], window: int = 1024) -> dict[str, float]:
    """Bits per UTF-8 byte over whole documents."""
    stride = window // 2
    nl = model.encode("\n")
    reqs, nbytes = [], 0
    for d in docs:
        ids = model.encode(d)
        nbytes += len(d.encode("utf-8"))
        reqs.append((nl, ids[:window]))
        for p in range(window, len(ids), stride):
            reqs.append((ids[p - stride:p], ids[p:p + stride]))
    s = model.loglikelihood_tokens(reqs)
    ntok = sum(x[2] for x in s)
    return {"bpb": -sum(x[0] for x in s) / math.log(2) / max(1, nbytes), "bytes_per_token": nbytes / max(1, ntok),
            "docs": len(docs)}


MC_TASKS: dict[str, Callable[[int | None], list[MCExample]]] = {
    "hellaswag": task_hellaswag,
    "arc_easy": lambda n: task_arc("ARC-Easy", n),
    "arc_challenge": lambda n: task_arc("ARC-Challenge", n),
    "piqa": task_piqa,
    "xstorycloze_en": lambda n: task_xstorycloze("en", n),
    "xstorycloze_zh": lambda n: task_xstorycloze("zh", n),
    "xcopa_zh": task_xcopa_zh,
}
OTHER_TASKS = ["winogrande", "lambada_openai", "bpb_wikitext2", "bpb_fineweb_edu_en", "bpb_fineweb_edu_zh",
               "bpb_wiki_zh"]
ALL_TASKS = [*MC_TASKS, *OTHER_TASKS]


def run_tasks(model: LogLikelihoodModel, tasks: Iterable[str], limit: int | None) -> dict[str, dict[str, float]]:
    results = {}
    for task in tasks:
        t0 = time.perf_counter()
        if task in MC_TASKS:
            m = score_multiple_choice(model, MC_TASKS[task](limit))
        elif task == "winogrande":
            m = eval_winogrande(model, limit)
        elif task == "lambada_openai":
            m = eval_lambada(model, limit)
        elif task.startswith("bpb_"):
            m = eval_bpb(model, bpb_documents(task[4:], limit))
        else:
            raise ValueError(f"unknown task {task!r}; known: {ALL_TASKS}")
        results[task] = m
        shown = " ".join(f"{k}={v:.4f}" if isinstance(v, float) else f"{k}={v}" for k, v in m.items())
        print(f"[{model.name}] {task}: {shown} ({time.perf_counter() - t0:.0f}s)", flush=True)
    return results


def main(argv: list[str] | None = None) -> None:
    global DATA_DIR
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--model", help="exported model directory")
    src.add_argument("--hf-model", help="HuggingFace causal LM id or path")
    ap.add_argument("--tasks", default=",".join(ALL_TASKS))
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--max-len", type=int, default=2048)
    ap.add_argument("--data-dir", default=None, help="local task copies (datasets.save_to_disk)")
    ap.add_argument("--output", default="eval_results.jsonl")
    args = ap.parse_args(argv)
    DATA_DIR = Path(args.data_dir) if args.data_dir else None
    model = MykModel(args.model, args.max_len) if args.model else HFModel(args.hf_model, args.max_len)
    print(f"model={model.name} params={model.num_params / 1e6:.1f}M")
    tasks = [t.strip() for t in args.tasks.split(",") if t.strip()]
    results = run_tasks(model, tasks, args.limit)
    with Path(args.output).open("a", encoding="utf-8") as f:
        f.write(json.dumps({"model": model.name, "params": model.num_params, "limit": args.limit,
                            "results": results}, ensure_ascii=False) + "\n")


if __name__ == "__main__":
    main()
