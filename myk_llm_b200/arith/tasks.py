"""Arithmetic problems rendered as character strings.

An example is ``<prompt>=<completion>$``: the model reads the prompt up to ``=`` and is
trained on, and must generate, the completion and the ``$`` end marker.  The answer is
what follows the last ``|`` of the completion (the whole completion without a chain of
thought).  Formats (the reference's ``src/myk_llm/arith/tasks.py`` defines the same
strings, so runs and their parsed answers are comparable):

* ``direct``:  ``123+456=579$``
* ``reverse``: ``123+456=975$`` (answer least-significant digit first)
* ``cot`` addition, one step per digit from the least significant, ``a+b+carry:ss``:
  ``123+456=3+6+0:09,2+5+0:07,1+4+0:05|579$``
* ``cot`` multiplication, partial products a*b_i*10^i and running sums written least
  significant first, then the answer: ``37*24=841;047>888|888$``

``reverse_operands`` writes the prompt operands least significant first; ``filler_prob``
inserts runs of ``_`` between prompt characters so digit offsets vary.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Literal

EOS, PAD, FILLER = "$", "#", "_"
# id 0 is padding; new characters are appended so existing ids never move
VOCAB = [PAD, EOS, *"0123456789", "+", "*", "=", "|", ":", ",", ";", ">", FILLER]


class CharTokenizer:
    def __init__(self) -> None:
        self.chars = list(VOCAB)
        self.index = {c: i for i, c in enumerate(self.chars)}
        self.pad_id, self.eos_id = self.index[PAD], self.index[EOS]
        self.digit_ids = [self.index[str(d)] for d in range(10)]

    def __len__(self) -> int:
        return len(self.chars)

    def encode(self, text: str) -> list[int]:
        return [self.index[c] for c in text]

    def decode(self, ids) -> str:
        return "".join(self.chars[i] for i in ids)


@dataclass
class TaskConfig:
    op: Literal["add", "mul"] = "add"
    format: Literal["direct", "reverse", "cot"] = "cot"
    min_digits: int = 1
    train_digits: int = 10  # each operand's length uniform in [min_digits, train_digits]
    reverse_operands: bool = False
    filler_prob: float = 0.0
    max_fillers: int = 3
    eval_digits: list[int] = field(default_factory=list)  # empty: 1 .. 2 * train_digits

    def eval_lengths(self) -> list[int]:
        return list(self.eval_digits) or list(range(1, 2 * self.train_digits + 1))


def _lsd_first(n: int) -> str:
    return str(n)[::-1]


def cot_addition(a: int, b: int) -> str:
    xa, xb = _lsd_first(a), _lsd_first(b)
    carry, parts = 0, []
    for i in range(max(len(xa), len(xb))):
        da = int(xa[i]) if i < len(xa) else 0
        db = int(xb[i]) if i < len(xb) else 0
        s = da + db + carry
        parts.append(f"{da}+{db}+{carry}:{s:02d}")
        carry = s // 10
    return ",".join(parts)


def cot_multiplication(a: int, b: int) -> str:
    parts, total = [], 0
    for i, d in enumerate(_lsd_first(b)):
        p = a * int(d)
        total += p * 10 ** i
        text = "0" * i + _lsd_first(p)
        parts.append(text if i == 0 else f"{text}>{_lsd_first(total)}")
    return ";".join(parts)


def true_answer(a: int, b: int, config: TaskConfig) -> int:
    return a + b if config.op == "add" else a * b


def render(a: int, b: int, config: TaskConfig) -> tuple[str, str]:
    """(prompt ending in '=', completion ending in EOS)."""
    sym = "+" if config.op == "add" else "*"
    x, y = (_lsd_first(a), _lsd_first(b)) if config.reverse_operands else (str(a), str(b))
    ans = true_answer(a, b, config)
    if config.format == "direct":
        comp = str(ans)
    elif config.format == "reverse":
        comp = _lsd_first(ans)
    else:
        steps = cot_addition(a, b) if config.op == "add" else cot_multiplication(a, b)
        comp = f"{steps}|{ans}"
    return f"{x}{sym}{y}=", comp + EOS


def add_fillers(prompt: str, rng: random.Random, prob: float, max_fillers: int) -> str:
    """Runs of FILLER before every prompt character but the first (with probability
    ``prob`` each)."""
    if prob <= 0:
        return prompt
    out = [prompt[0]]
    for ch in prompt[1:]:
        if rng.random() < prob:
            out.append(FILLER * rng.randint(1, max_fillers))
        out.append(ch)
    return "".join(out)


def parse_answer(completion: str, config: TaskConfig) -> int | None:
    text = completion.split(EOS, 1)[0].rsplit("|", 1)[-1]
    if config.format == "reverse":
        text = text[::-1]
    return int(text) if text.isdigit() else None


def sample_operand(rng: random.Random, digits: int) -> int:
    lo = 10 ** (digits - 1) if digits > 1 else 0
    return rng.randint(lo, 10 ** digits - 1)


def sample_problem(rng: random.Random, config: TaskConfig) -> tuple[int, int]:
    da = rng.randint(config.min_digits, config.train_digits)
    db = rng.randint(config.min_digits, config.train_digits)
    return sample_operand(rng, da), sample_operand(rng, db)
