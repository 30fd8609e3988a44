"""The arithmetic testbed's model: the language model plus an optional Abacus digit-position
embedding, greedy completion, and exact-match evaluation per operand length.

Greedy completion groups prompts of equal token length, prefills each group once and then
decodes one character per step from the model's per-layer caches (positions advance
together inside a group, so no padding is ever attended to); a row that produced the end
marker stops being written.
"""

from __future__ import annotations

import random
from collections import defaultdict
from dataclasses import dataclass

import torch
import torch.nn as nn

from ..data.config import Batch
from ..models import ModelConfig, MykLLM
from ..utils.testbed import autocast_for
from .tasks import EOS, CharTokenizer, TaskConfig, add_fillers, parse_answer, render, sample_operand, true_answer


@dataclass
class DigitEmbeddingConfig:
    """Abacus embedding (McLeish et al., 2024): a learned vector per digit position inside
    its number (1 = the first digit written).  Training shifts the positions by a random
    offset in [0, max_offset] so that positions past the training lengths get trained."""

    enabled: bool = False
    max_offset: int = 50
    max_index: int = 128


def digit_indices(input_ids: torch.Tensor, digit_ids: torch.Tensor) -> torch.Tensor:
    """1-based position of every digit inside its run of consecutive digits, 0 for other
    characters (causal: depends only on earlier characters)."""
    digit = torch.isin(input_ids, digit_ids)
    run = digit.long().cumsum(1)
    # the count of digits before the current run: the running total at its last non-digit
    before = torch.where(digit, torch.zeros_like(run), run).cummax(1).values
    return (run - before) * digit


class ArithModel(nn.Module):
    def __init__(self, config: ModelConfig, digits: DigitEmbeddingConfig) -> None:
        super().__init__()
        self.lm = MykLLM(config)
        self.digits = digits
        self.tokenizer = CharTokenizer()
        if config.vocab_size < len(self.tokenizer):
            raise ValueError(f"model.vocab_size must be at least {len(self.tokenizer)}")
        self.register_buffer("digit_ids", torch.tensor(self.tokenizer.digit_ids), persistent=False)
        self.digit_embed = None
        if digits.enabled:
            self.digit_embed = nn.Embedding(digits.max_index + digits.max_offset + 1, config.hidden_size)
            with torch.no_grad():
                self.digit_embed.weight.normal_(0.0, config.initializer_range)
                self.digit_embed.weight[0] = 0.0  # non-digits add nothing

    def embed_offset(self, input_ids: torch.Tensor, random_offset: bool, last: int = 0) -> torch.Tensor | None:
        """Digit-position vectors for ``input_ids`` (only its last ``last`` columns if set)."""
        if self.digit_embed is None:
            return None
        index = digit_indices(input_ids, self.digit_ids)
        if last:
            index = index[:, -last:]
        if random_offset and self.digits.max_offset:
            shift = torch.randint(0, self.digits.max_offset + 1, (index.shape[0], 1), device=index.device)
            index = torch.where(index > 0, index + shift, index)
        return self.digit_embed(index.clamp(max=self.digit_embed.num_embeddings - 1))

    def forward(self, batch: Batch, head):
        return self.lm(batch.input_ids, seqlens=batch.seqlens, head=head,
                       embed_offset=self.embed_offset(batch.input_ids, random_offset=self.training))

    @torch.no_grad()
    def _complete_group(self, rows: torch.Tensor, steps: int) -> torch.Tensor:
        """Greedy continuation of equal-length prompts (n, p): (n, p + steps) ids."""
        tok, dev = self.tokenizer, rows.device
        n, p = rows.shape
        ids = torch.cat([rows, torch.full((n, steps), tok.pad_id, dtype=rows.dtype, device=dev)], 1)
        done = torch.zeros(n, dtype=torch.bool, device=dev)
        allowed = len(tok)  # never pick ids past the character set
        with autocast_for(dev):
            out = self.lm(rows, use_cache=True, embed_offset=self.embed_offset(rows, False))
            for t in range(steps):
                nxt = self.lm.logits(out.hidden[:, -1])[:, :allowed].argmax(-1)
                ids[:, p + t] = torch.where(done, torch.full_like(nxt, tok.pad_id), nxt)
                done |= nxt == tok.eos_id
                if bool(done.all()) or t + 1 == steps:
                    break
                cur = ids[:, p + t:p + t + 1]
                pos = torch.full((n, 1), p + t, dtype=torch.long, device=dev)
                out = self.lm(cur, position_ids=pos, cache=out.cache, use_cache=True,
                              embed_offset=self.embed_offset(ids[:, :p + t + 1], False, last=1))
        return ids

    @torch.no_grad()
    def greedy_complete(self, prompts: list[str], max_new_tokens: int) -> list[str]:
        tok, dev = self.tokenizer, self.digit_ids.device
        groups: dict[int, list[int]] = defaultdict(list)
        for i, p in enumerate(prompts):
            groups[len(p)].append(i)
        out: list[str] = [""] * len(prompts)
        for length, members in groups.items():
            rows = torch.tensor([tok.encode(prompts[i]) for i in members], dtype=torch.long, device=dev)
            done = self._complete_group(rows, max_new_tokens)[:, length:].tolist()
            for i, gen in zip(members, done):
                text = tok.decode(gen)
                out[i] = text[:text.index(EOS) + 1] if EOS in text else text
        return out


def completion_budget(task: TaskConfig, digits: int) -> int:
    """Characters to generate for operands of ``digits`` digits (the longest completion + 4)."""
    largest = 10 ** digits - 1
    return len(render(largest, largest, task)[1]) + 4


@torch.no_grad()
def evaluate_lengths(model: ArithModel, task: TaskConfig, lengths: list[int], examples: int, seed: int,
                     batch_size: int = 512, fillers: bool = False) -> dict[int, float]:
    """Exact-match accuracy of the final answer (with the end marker) for both operands of
    ``d`` digits, per ``d``."""
    training = model.training
    model.eval()
    rng = random.Random(seed)
    scores: dict[int, float] = {}
    for d in lengths:
        problems = [(sample_operand(rng, d), sample_operand(rng, d)) for _ in range(examples)]
        prompts = [render(a, b, task)[0] for a, b in problems]
        if fillers:
            prompts = [add_fillers(p, rng, task.filler_prob, task.max_fillers) for p in prompts]
        budget = completion_budget(task, d)
        right = 0
        for lo in range(0, examples, batch_size):
            for text, (a, b) in zip(model.greedy_complete(prompts[lo:lo + batch_size], budget),
                                    problems[lo:lo + batch_size]):
                right += text.endswith(EOS) and parse_answer(text, task) == true_answer(a, b, task)
        scores[d] = right / examples
    model.train(training)
    return scores
