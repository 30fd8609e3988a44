"""Arithmetic problems as character strings.

An example is ``<prompt>=<completion>$``: the model reads the prompt (through ``=``), is
trained on the completion and the ``$`` end marker, and must generate them.  The answer is
the text after the completion's last ``|`` (all of it when there is no chain of thought).
The formats are an interface shared with the reference's ``src/myk_llm/arith/tasks.py``
(the same strings, so runs and their parsed answers compare):

* ``direct``:  ``123+456=579$``
* ``reverse``: ``123+456=975$`` (the answer least-significant digit first)
* ``cot`` addition: one step per digit from the least significant, ``a+b+carry:ss``:
  ``123+456=3+6+0:09,2+5+0:07,1+4+0:05|579$``
* ``cot`` multiplication: each partial product ``a * b_i * 10^i`` written least
  significant first, after the first one followed by ``>`` and the running sum (also
  least significant first), then the answer: ``37*24=841;047>888|888$``

``reverse_operands`` writes the prompt's operands least significant first; ``filler_prob``
puts runs of ``_`` between prompt characters so digits move to varying offsets.

Here numbers are handled as little-endian digit lists (``digits_of``), from which every
format is assembled.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Literal

EOS, PAD, FILLER = "$", "#", "_"
# character set; id 0 is padding and new characters go at the end so ids never move
VOCAB = [PAD, EOS, *"0123456789", "+", "*", "=", "|", ":", ",", ";", ">", FILLER]
OPS = {"add": ("+", lambda a, b: a + b), "mul": ("*", lambda a, b: a * b)}


class CharTokenizer:
    """One id per character of ``VOCAB``."""

    def __init__(self) -> None:
        self.chars = list(VOCAB)
        self.index = {ch: i for i, ch in enumerate(self.chars)}
        self.pad_id, self.eos_id = self.index[PAD], self.index[EOS]
        self.digit_ids = [self.index[d] for d in "0123456789"]

    def __len__(self) -> int:
        return len(self.chars)

    def encode(self, text: str) -> list[int]:
        return [self.index[ch] for ch in text]

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
        return list(self.eval_digits) if self.eval_digits else list(range(1, 2 * self.train_digits + 1))


def digits_of(n: int) -> list[int]:
    """Little-endian decimal digits (``0`` -> ``[0]``)."""
    out = []
    while True:
        n, d = divmod(n, 10)
        out.append(d)
        if n == 0:
            return out


def little_endian(n: int) -> str:
    return "".join(map(str, digits_of(n)))


def cot_addition(a: int, b: int) -> str:
    da, db = digits_of(a), digits_of(b)
    width = max(len(da), len(db))
    da, db = da + [0] * (width - len(da)), db + [0] * (width - len(db))
    steps, carry = [], 0
    for x, y in zip(da, db):
        total = x + y + carry
        steps.append(f"{x}+{y}+{carry}:{total // 10}{total % 10}")
        carry = total // 10
    return ",".join(steps)


def cot_multiplication(a: int, b: int) -> str:
    steps, running = [], 0
    for place, digit in enumerate(digits_of(b)):
        partial = a * digit * 10 ** place
        running += partial
        # the partial product shifted by `place`, written least significant first
        text = "0" * place + little_endian(a * digit)
        steps.append(text if place == 0 else f"{text}>{little_endian(running)}")
    return ";".join(steps)


def true_answer(a: int, b: int, config: TaskConfig) -> int:
    return OPS[config.op][1](a, b)


def _completion(a: int, b: int, config: TaskConfig) -> str:
    answer = true_answer(a, b, config)
    if config.format == "direct":
        return str(answer)
    if config.format == "reverse":
        return little_endian(answer)
    chain = cot_addition(a, b) if config.op == "add" else cot_multiplication(a, b)
    return f"{chain}|{answer}"


def render(a: int, b: int, config: TaskConfig) -> tuple[str, str]:
    """(prompt ending in ``=``, completion ending in ``$``)."""
    write = little_endian if config.reverse_operands else str
    return f"{write(a)}{OPS[config.op][0]}{write(b)}=", _completion(a, b, config) + EOS


def add_fillers(prompt: str, rng: random.Random, prob: float, max_fillers: int) -> str:
    """With probability ``prob`` per position, a run of 1..max_fillers ``_`` before each
    prompt character but the first."""
    if prob <= 0:
        return prompt
    pieces = [prompt[0]]
    for ch in prompt[1:]:
        if rng.random() < prob:
            pieces.append(FILLER * rng.randint(1, max_fillers))
        pieces.append(ch)
    return "".join(pieces)


def parse_answer(completion: str, config: TaskConfig) -> int | None:
    """The integer answer of a generated completion (None if it is not a number)."""
    body = completion.split(EOS)[0]
    text = body[body.rfind("|") + 1:]
    if config.format == "reverse":
        text = text[::-1]
    return int(text) if text.isdigit() else None


def sample_operand(rng: random.Random, digits: int) -> int:
    """A uniform number with exactly ``digits`` digits (0..9 for one digit)."""
    return rng.randint(0 if digits == 1 else 10 ** (digits - 1), 10 ** digits - 1)


def sample_problem(rng: random.Random, config: TaskConfig) -> tuple[int, int]:
    lengths = [rng.randint(config.min_digits, config.train_digits) for _ in range(2)]
    return sample_operand(rng, lengths[0]), sample_operand(rng, lengths[1])
