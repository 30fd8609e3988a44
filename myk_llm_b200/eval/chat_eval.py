"""Generation sanity check for chat (SFT) models: a fixed English / Chinese prompt set
under several decoding settings, scored with cheap automatic signals, every reply kept.

Signals per reply (the reference's ``src/myk_llm/eval/chat_eval.py:39-160`` reports the
same five):

* ``stop``: the end-of-turn token came before the token budget ran out;
* ``rep4``: fraction of repeated token 4-grams (looping);
* ``lang_ok``: the reply is mostly in the prompt's language (CJK share of letters);
* ``leak``: the reply starts a new turn by itself (``<|im_start|>`` or a role line);
* ``hit``: for prompts with a known answer, the reply contains one of the answers.

    python -m myk_llm_b200.eval.chat_eval runs/200m-sft/export --output chat_eval.jsonl
"""

from __future__ import annotations

import argparse
import json
import re
from collections import defaultdict
from dataclasses import dataclass, field
from pathlib import Path

import torch


@dataclass
class ChatCase:
    turns: list[str]  # user turns; earlier ones are answered by the model itself
    lang: str  # "en" | "zh"
    answers: list[str] = field(default_factory=list)


CASES: list[ChatCase] = [
    ChatCase(["What is the largest planet in our solar system?"], "en", ["Jupiter"]),
    ChatCase(["What is 9 minus 3?"], "en", ["6", "six"]),
    ChatCase(["What is the opposite of 'hot'?"], "en", ["cold"]),
    ChatCase(["How many legs does a spider have?"], "en", ["8", "eight"]),
    ChatCase(["Which ocean lies between Europe and North America?"], "en", ["Atlantic"]),
    ChatCase(["What gas do plants take in from the air to make food?"], "en", ["carbon dioxide", "CO2"]),
    ChatCase(["Translate to English: 今天天气很好。"], "en", ["weather"]),
    ChatCase(["日本的首都是哪里？"], "zh", ["东京"]),
    ChatCase(["10减去4等于几？"], "zh", ["6", "六"]),
    ChatCase(["一天有多少个小时？"], "zh", ["24", "二十四"]),
    ChatCase(["地球围绕什么天体公转？"], "zh", ["太阳"]),
    ChatCase(["《西游记》的作者是谁？"], "zh", ["吴承恩"]),
    ChatCase(["把这句话翻译成中文：The cat is sleeping."], "zh", ["猫"]),
    ChatCase(["冰融化后变成什么？"], "zh", ["水"]),
    ChatCase(["Please describe yourself in one short paragraph."], "en"),
    ChatCase(["Explain in simple words why the moon has phases."], "en"),
    ChatCase(["List three ways to save water at home, as a numbered list."], "en"),
    ChatCase(["Write a four-line poem about mountains."], "en"),
    ChatCase(["Write a Python function that reverses a string."], "en"),
    ChatCase(["请用两句话介绍一下你自己。"], "zh"),
    ChatCase(["用通俗的语言解释一下什么是神经网络。"], "zh"),
    ChatCase(["列出三个保持健康的好习惯。"], "zh"),
    ChatCase(["写一首关于春天的短诗。"], "zh"),
    ChatCase(["为什么天空在傍晚会变红？简单说明。"], "zh"),
    ChatCase(["I live in Berlin and work as a baker.", "Which city do I live in?"], "en", ["Berlin"]),
    ChatCase(["我最喜欢的水果是香蕉。", "我最喜欢什么水果？"], "zh", ["香蕉"]),
]

DECODING = {
    "greedy": dict(temperature=0.0, top_k=None, repetition_penalty=1.0),
    "sample": dict(temperature=0.7, top_k=50, repetition_penalty=1.0),
    "chat_default": dict(temperature=0.7, top_k=50, top_p=0.95, repetition_penalty=1.1),
}

_CJK = re.compile(r"[一-鿿]")
_LATIN = re.compile(r"[A-Za-z]")


def reply_language_ok(text: str, lang: str) -> bool:
    """Mostly Chinese for ``zh``, mostly Latin script for ``en`` (a CJK character counts
    as a word; about four Latin letters make one)."""
    cjk, latin = len(_CJK.findall(text)), len(_LATIN.findall(text))
    if cjk + latin == 0:
        return True
    share = cjk / (cjk + latin / 4)
    return share >= 0.5 if lang == "zh" else share < 0.5


def contains_answer(text: str, answer: str) -> bool:
    if answer.isdigit():  # whole numbers only: "6" must not hit "16"
        return re.search(rf"(?<!\d){answer}(?!\d)", text) is not None
    return answer.lower() in text.lower()


def repeated_ngram_fraction(tokens: list[int], n: int = 4) -> float:
    grams = [tuple(tokens[i:i + n]) for i in range(len(tokens) - n + 1)]
    return 0.0 if not grams else 1.0 - len(set(grams)) / len(grams)


def leaked_turn(ids: list[int], text: str, im_start: int | None) -> bool:
    return (im_start is not None and im_start in ids) or bool(re.search(r"(^|\n)(user|assistant)\n", text))


def evaluate(model, tokenizer, decodings: list[str], max_tokens: int = 256, seed: int = 0,
             cases: list[ChatCase] = CASES, model_name: str = "") -> list[dict]:
    from ..chat import build_prompt_ids, generate_reply

    im_start = tokenizer.convert_tokens_to_ids("<|im_start|>")
    records = []
    for dname in decodings:
        dec = DECODING[dname]
        for ci, case in enumerate(cases):
            history: list[tuple[str, str]] = []
            text, ids, stopped = "", [], False
            for user in case.turns:
                torch.manual_seed(seed + ci)
                prompt = build_prompt_ids(model, tokenizer, history, user, raw=False)
                text, ids, stopped = generate_reply(model, tokenizer, prompt, max_tokens, **dec)
                history.append((user, text))
            records.append({"model": model_name, "decoding": dname, "case": ci, "turns": case.turns,
                            "lang": case.lang, "reply": text, "stop": stopped,
                            "rep4": repeated_ngram_fraction(ids), "lang_ok": reply_language_ok(text, case.lang),
                            "leak": leaked_turn(ids, text, im_start),
                            "hit": any(contains_answer(text, a) for a in case.answers) if case.answers else None,
                            "num_tokens": len(ids)})
    return records


def summarize(records: list[dict]) -> dict[str, dict[str, float]]:
    by = defaultdict(list)
    for r in records:
        by[r["decoding"]].append(r)
    out = {}
    for name, rs in by.items():
        hits = [r["hit"] for r in rs if r["hit"] is not None]
        out[name] = {"stop": sum(r["stop"] for r in rs) / len(rs), "rep4": sum(r["rep4"] for r in rs) / len(rs),
                     "lang_ok": sum(r["lang_ok"] for r in rs) / len(rs), "leak": sum(r["leak"] for r in rs) / len(rs),
                     "hit": sum(hits) / max(1, len(hits))}
    return out


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("model", help="exported model directory")
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--decoding", default=",".join(DECODING))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--output", default="chat_eval.jsonl")
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    from ..models.io import load_model

    model = load_model(args.model, device="cuda" if torch.cuda.is_available() else "cpu").eval()
    tok = AutoTokenizer.from_pretrained(args.model)
    with torch.no_grad():
        recs = evaluate(model, tok, [d.strip() for d in args.decoding.split(",")], args.max_tokens, args.seed,
                        model_name=args.model)
    with Path(args.output).open("a", encoding="utf-8") as f:
        for r in recs:
            f.write(json.dumps(r, ensure_ascii=False) + "\n")
    for name, m in summarize(recs).items():
        print(f"{name}: " + " ".join(f"{k}={v:.3f}" for k, v in m.items()))


if __name__ == "__main__":
    main()
