"""Retrieval examples over a small token vocabulary.

One example is one sequence: records scattered among noise tokens, then queries.  Each
of N items is a chain of h hops through distinct keys (h = 1: a key -> value record;
h > 1: variable tracking)::

    records  k0 k1 ;  k1 k2 ;  k2 v v v v ;          (h = 3, keys key_len tokens long)
    query    ? k0  ->  v v v v $                      (cot: k1 k2 v v v v $)

A query ends with the key itself, so an induction head (find the earlier occurrence of
the current tokens, copy what follows) can answer it.  Keys, values and noise use
disjoint alphabets and record parts have fixed lengths, so records need no separators
inside.  All records are shuffled and dropped at random positions in the noise; Q of
the N items are queried at the end; only the answers (with ``$``) are supervised.

Regimes: ``needle`` (few items, mostly noise) and ``capacity`` (many items, little noise;
``scale_records`` keeps the load per token when evaluating longer contexts).

Token layout (shared with the reference's ``src/myk_llm/lc/tasks.py`` so that trained
checkpoints and examples are interchangeable): PAD 0, EOS 1, QUERY 2, SEP 3, keys
16..143, values 144..207, noise 208..463 (464 ids).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

import numpy as np

PAD, EOS, QUERY, SEP = 0, 1, 2, 3
KEY_BASE, KEY_SYMBOLS = 16, 128
VALUE_BASE, VALUE_SYMBOLS = KEY_BASE + KEY_SYMBOLS, 64
NOISE_BASE, NOISE_SYMBOLS = VALUE_BASE + VALUE_SYMBOLS, 256
VOCAB_SIZE = NOISE_BASE + NOISE_SYMBOLS


@dataclass
class TaskConfig:
    min_len: int = 256            # training example lengths in [min_len, max_len]
    max_len: int = 2048           # also the packed row length
    length_dist: Literal["uniform", "log_uniform"] = "uniform"
    num_records: int = 8          # items per example (at max_len when scale_records)
    min_records: int = 0          # >0: training draws the item count in [min_records, num_records]
    copy_fraction: float = 0.0    # share of copy examples (span, then the span again)
    copy_min: int = 16
    copy_max: int = 128
    scale_records: bool = False
    num_queries: int = 4
    key_len: int = 2
    value_len: int = 4
    hops: list[int] = field(default_factory=lambda: [1])
    eval_hops: list[int] = field(default_factory=list)
    cot: bool = False
    eval_lengths: list[int] = field(default_factory=lambda: [512, 1024, 2048, 4096, 8192, 16384, 32768, 65536])
    depth_buckets: int = 10

    def __post_init__(self) -> None:
        if not 0 < self.min_len <= self.max_len:
            raise ValueError("need 0 < min_len <= max_len")
        if self.num_queries > self.num_records:
            raise ValueError("num_queries must not exceed num_records (queried items are distinct)")
        if not 0 <= self.min_records <= self.num_records:
            raise ValueError("need 0 <= min_records <= num_records")
        if self.copy_fraction and not 1 <= self.copy_min <= self.copy_max <= self.max_len // 2:
            raise ValueError("need 1 <= copy_min <= copy_max <= max_len / 2")
        if not self.hops or min(self.hops) < 1 or (self.eval_hops and min(self.eval_hops) < 1):
            raise ValueError("hop counts must be positive")

    def sample_length(self, rng: np.random.Generator) -> int:
        if self.length_dist == "uniform":
            return int(rng.integers(self.min_len, self.max_len + 1))
        return int(np.exp(rng.uniform(np.log(self.min_len), np.log(self.max_len + 1))))

    def records_at(self, length: int, count: int | None = None) -> int:
        c = self.num_records if count is None else count
        return max(1, round(c * length / self.max_len)) if self.scale_records else c

    def sample_records(self, rng: np.random.Generator) -> int | None:
        return int(rng.integers(self.min_records, self.num_records + 1)) if self.min_records else None


@dataclass
class Example:
    ids: np.ndarray                  # (length,) int64
    answers: list[tuple[int, int]]   # [start, end) of every query's answer in ids
    depths: list[float]              # first record of the queried item / context length
    hops: list[int]


def _keys(rng: np.random.Generator, count: int, key_len: int) -> list[list[int]]:
    """``count`` distinct keys of ``key_len`` key symbols: distinct integers below
    ``KEY_SYMBOLS ** key_len`` written in base ``KEY_SYMBOLS``, most significant first."""
    space = KEY_SYMBOLS ** key_len
    if count > space:
        raise ValueError(f"{count} keys needed, only {space} exist; raise key_len")
    codes = rng.choice(space, size=count, replace=False)
    symbols = np.empty((count, key_len), dtype=np.int64)
    for j in range(key_len - 1, -1, -1):
        codes, symbols[:, j] = np.divmod(codes, KEY_SYMBOLS)
    return (symbols + KEY_BASE).tolist()


@dataclass
class _Item:
    chain: list[list[int]]   # the keys of its hops, in order
    value: list[int]

    def records(self) -> list[list[int]]:
        """``k_i k_{i+1} ;`` for each hop, then ``k_last v... ;``."""
        links = [a + b + [SEP] for a, b in zip(self.chain, self.chain[1:])]
        return links + [self.chain[-1] + self.value + [SEP]]

    def query(self, cot: bool) -> tuple[list[int], list[int]]:
        """(prompt ``? k_0``, answer: the later keys when ``cot``, the value, ``$``)."""
        middle = [t for key in self.chain[1:] for t in key] if cot else []
        return [QUERY] + self.chain[0], middle + self.value + [EOS]


class _Layout:
    """Writes records at random offsets into noise, then the queries, into one array."""

    def __init__(self, length: int) -> None:
        self.ids = np.empty(length, dtype=np.int64)
        self.pos = 0

    def put(self, tokens) -> int:
        start = self.pos
        self.ids[start:start + len(tokens)] = tokens
        self.pos += len(tokens)
        return start


def make_example(rng: np.random.Generator, task: TaskConfig, length: int, records: int | None = None) -> Example:
    """One example of exactly ``length`` tokens.  The order of random draws (hop counts,
    keys, values, queried items, record order, gaps, noise) is fixed, so a seed gives the
    same example as the reference's generator."""
    n = task.records_at(length, records)
    hops = rng.choice(task.hops, size=n)
    keys = _keys(rng, int(hops.sum()), task.key_len)
    values = (rng.integers(0, VALUE_SYMBOLS, size=(n, task.value_len)) + VALUE_BASE).tolist()
    bounds = np.concatenate(([0], np.cumsum(hops))).tolist()
    items = [_Item(keys[bounds[i]:bounds[i + 1]], values[i]) for i in range(n)]
    recs = [(i, r) for i, item in enumerate(items) for r in item.records()]
    queried = rng.choice(n, size=min(task.num_queries, n), replace=False).tolist()
    queries = [items[i].query(task.cot) for i in queried]
    context = length - sum(len(p) + len(a) for p, a in queries)
    noise = context - sum(len(r) for _, r in recs)
    if noise < 0:
        raise ValueError(f"{n} items and their queries do not fit in {length} tokens")
    order = rng.permutation(len(recs)).tolist()
    gaps = np.sort(rng.integers(0, noise + 1, size=len(recs))).tolist()  # noise tokens before each record
    filler = rng.integers(NOISE_BASE, NOISE_BASE + NOISE_SYMBOLS, size=noise)
    out = _Layout(length)
    first_seen = [context] * n
    taken = 0
    for r, gap in zip(order, gaps):
        out.put(filler[taken:gap])
        taken = gap
        item, tokens = recs[r]
        first_seen[item] = min(first_seen[item], out.put(tokens))
    out.put(filler[taken:])
    answers = []
    for prompt, answer in queries:
        out.put(prompt)
        start = out.put(answer)
        answers.append((start, start + len(answer)))
    return Example(out.ids, answers, [first_seen[i] / context for i in queried], [int(hops[i]) for i in queried])


def make_copy_example(rng: np.random.Generator, task: TaskConfig) -> Example:
    """A random span followed by the same span; the repeat after its first token is the answer."""
    width = int(rng.integers(task.copy_min, task.copy_max + 1))
    span = rng.integers(KEY_BASE, VOCAB_SIZE, size=width)
    return Example(np.concatenate([span, span]), [(width + 1, 2 * width)], [0.0], [0])


def resolve(ids: np.ndarray, query_key: list[int], key_len: int) -> list[int]:
    """Follow the context's records from ``query_key`` to its value: a direct statement of
    the task used by the tests.  A record starts with a key symbol right after a
    separator, a noise token or the beginning."""
    toks = ids.tolist()
    toks = toks[:toks.index(QUERY)]
    lookup: dict[tuple[int, ...], list[int]] = {}
    i = 0
    while i < len(toks):
        boundary = i == 0 or toks[i - 1] == SEP or toks[i - 1] >= NOISE_BASE
        if KEY_BASE <= toks[i] < VALUE_BASE and boundary:
            end = toks.index(SEP, i)
            lookup[tuple(toks[i:i + key_len])] = toks[i + key_len:end]
            i = end + 1
        else:
            i += 1
    target = lookup[tuple(query_key)]
    while all(KEY_BASE <= t < VALUE_BASE for t in target):  # a link to the next key
        target = lookup[tuple(target)]
    return target
