"""The language model plus an optional Abacus digit-position embedding, and batched
greedy exact-match evaluation per operand length."""

from __future__ import annotations

import contextlib
import random
from dataclasses import dataclass

import torch
import torch.nn as nn

from ..data.config import Batch
from ..models import MykLLM, ModelConfig
from .tasks import EOS, CharTokenizer, TaskConfig, add_fillers, parse_answer, render, sample_operand, true_answer


@dataclass
class DigitEmbeddingConfig:
    """Abacus embedding (McLeish et al., 2024): a learned vector per digit index within
    its number (1 = first digit written).  Training adds a random offset in
    [0, max_offset] so indices past the training lengths are trained too."""

    enabled: bool = False
    max_offset: int = 50
    max_index: int = 128


def digit_indices(input_ids: torch.Tensor, digit_ids: torch.Tensor) -> torch.Tensor:
    """1-based index of every digit inside its run of digits, 0 elsewhere (causal)."""
    is_d = torch.isin(input_ids, digit_ids)
    count = is_d.long().cumsum(1)
    start = torch.where(is_d, torch.zeros_like(count), count).cummax(1).values
    return torch.where(is_d, count - start, torch.zeros_like(count))


def _autocast(device: torch.device):
    return torch.autocast("cuda", dtype=torch.bfloat16) if device.type == "cuda" else contextlib.nullcontext()


class ArithModel(nn.Module):
    def __init__(self, config: ModelConfig, digits: DigitEmbeddingConfig) -> None:
        super().__init__()
        self.lm = MykLLM(config)
        self.digits = digits
        self.tokenizer = CharTokenizer()
        if len(self.tokenizer) > config.vocab_size:
            raise ValueError(f"model.vocab_size must be at least {len(self.tokenizer)}")
        self.register_buffer("digit_ids", torch.tensor(self.tokenizer.digit_ids), persistent=False)
        self.digit_embed = None
        if digits.enabled:
            self.digit_embed = nn.Embedding(digits.max_index + digits.max_offset + 1, config.hidden_size)
            nn.init.normal_(self.digit_embed.weight, std=config.initializer_range)
            with torch.no_grad():
                self.digit_embed.weight[0].zero_()

    def embed_offset(self, input_ids: torch.Tensor, random_offset: bool) -> torch.Tensor | None:
        if self.digit_embed is None:
            return None
        idx = digit_indices(input_ids, self.digit_ids)
        if random_offset and self.digits.max_offset:
            off = torch.randint(0, self.digits.max_offset + 1, (input_ids.size(0), 1), device=input_ids.device)
            idx = torch.where(idx > 0, idx + off, idx)
        return self.digit_embed(idx.clamp(max=self.digit_embed.num_embeddings - 1))

    def forward(self, batch: Batch, head):
        return self.lm(batch.input_ids, seqlens=batch.seqlens, head=head,
                       embed_offset=self.embed_offset(batch.input_ids, random_offset=self.training))

    @torch.no_grad()
    def greedy_complete(self, prompts: list[str], max_new_tokens: int) -> list[str]:
        """Greedy completions.  Each step re-runs the right-padded prefixes (causal, so
        padding never reaches real positions); finished rows leave the batch."""
        tok, dev = self.tokenizer, self.digit_ids.device
        lens = torch.tensor([len(p) for p in prompts], device=dev)
        buf = torch.full((len(prompts), int(lens.max()) + max_new_tokens), tok.pad_id, dtype=torch.long, device=dev)
        for r, p in enumerate(prompts):
            buf[r, :len(p)] = torch.tensor(tok.encode(p), device=dev)
        live = torch.arange(len(prompts), device=dev)
        for _ in range(max_new_tokens):
            if live.numel() == 0:
                break
            width = int(lens[live].max())
            ids = buf[live, :width]
            with _autocast(dev):
                hidden = self.lm(ids, embed_offset=self.embed_offset(ids, random_offset=False)).hidden
            last = hidden[torch.arange(live.numel(), device=dev), lens[live] - 1]
            nxt = self.lm.logits(last)[:, :len(tok)].argmax(-1)  # never ids past the character set
            buf[live, lens[live]] = nxt
            lens[live] += 1
            live = live[nxt != tok.eos_id]
        return [tok.decode(buf[r, len(p):int(lens[r])].tolist()) for r, p in enumerate(prompts)]


def completion_budget(task: TaskConfig, digits: int) -> int:
    top = 10 ** digits - 1
    return len(render(top, top, task)[1]) + 4


@torch.no_grad()
def evaluate_lengths(model: ArithModel, task: TaskConfig, lengths: list[int], examples: int, seed: int,
                     batch_size: int = 512, fillers: bool = False) -> dict[int, float]:
    """Exact-match accuracy of the final answer with both operands ``d`` digits long."""
    was = model.training
    model.eval()
    rng = random.Random(seed)
    acc = {}
    for d in lengths:
        probs = [(sample_operand(rng, d), sample_operand(rng, d)) for _ in range(examples)]
        budget = completion_budget(task, d)
        ok = 0
        for s in range(0, examples, batch_size):
            chunk = probs[s:s + batch_size]
            prompts = [render(a, b, task)[0] for a, b in chunk]
            if fillers:
                prompts = [add_fillers(p, rng, task.filler_prob, task.max_fillers) for p in prompts]
            for c, (a, b) in zip(model.greedy_complete(prompts, budget), chunk):
                ok += int(c.endswith(EOS) and parse_answer(c, task) == true_answer(a, b, task))
        acc[d] = ok / examples
    model.train(was)
    return acc
