"""Autoregressive sampling with per-layer caches: the simple eager loop behind ``generate``.

Contract (the reference's, ``src/myk_llm/model/generation.py:16-84``): the prompt is
prefilled with ``keep_last=1`` and the output head run on the last position only, then
tokens are produced one at a time; greedy when ``temperature <= 0``, else temperature,
top-k and top-p (nucleus) sampling after a CTRL-style repetition penalty over the tokens
generated so far (not the prompt); a row that emitted ``eos_token_id`` keeps emitting it,
and the loop stops once every row has.

The serving path (static caches, CUDA graphs, MTP speculative decoding) is
:mod:`myk_llm_b200.infer`.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .transformer import ModelOutput, MykLLM


def _head_last(model: MykLLM, output: ModelOutput):
    return output, model.logits(output.hidden[:, -1]).float()


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_k: int | None = None
    top_p: float | None = None
    repetition_penalty: float = 1.0

    def pick(self, logits: torch.Tensor, generated: torch.Tensor | None) -> torch.Tensor:
        """Next token per row from fp32 logits (batch, vocab)."""
        if generated is not None and generated.numel() and self.repetition_penalty != 1.0:
            logits = penalize_repeats(logits, generated, self.repetition_penalty)
        return sample(logits, self.temperature, self.top_k, self.top_p)


def penalize_repeats(logits: torch.Tensor, seen: torch.Tensor, penalty: float) -> torch.Tensor:
    """Divide positive (multiply negative) logits of already generated tokens by ``penalty``."""
    hit = torch.zeros_like(logits, dtype=torch.bool).scatter_(1, seen, True)
    scaled = torch.where(logits > 0, logits / penalty, logits * penalty)
    return torch.where(hit, scaled, logits)


def sample(logits: torch.Tensor, temperature: float, top_k: int | None, top_p: float | None) -> torch.Tensor:
    if temperature <= 0.0:
        return logits.argmax(dim=-1)
    z = logits / temperature
    if top_k is not None and top_k < z.shape[-1]:
        kth = z.topk(top_k, dim=-1).values[..., -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    if top_p is not None and top_p < 1.0:
        ranked, order = z.sort(dim=-1, descending=True)
        p = ranked.softmax(-1)
        outside = (p.cumsum(-1) - p) > top_p  # tokens whose predecessors already cover top_p
        z = z.scatter(-1, order, ranked.masked_fill(outside, float("-inf")))
    return torch.multinomial(F.softmax(z, dim=-1), 1).squeeze(-1)


@torch.no_grad()
def generate(model: MykLLM, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
             top_k: int | None = None, top_p: float | None = None, repetition_penalty: float = 1.0,
             eos_token_id: int | None = None) -> torch.Tensor:
    if input_ids.dim() != 2 or input_ids.shape[1] == 0:
        raise ValueError("input_ids must be a non-empty (batch, seq_len) tensor")
    prompt_len = input_ids.shape[1]
    if prompt_len + max_new_tokens > model.config.max_seq_len:
        raise ValueError(f"prompt ({prompt_len}) + max_new_tokens ({max_new_tokens}) exceeds max_seq_len "
                         f"{model.config.max_seq_len}")
    params = SamplingParams(temperature, top_k, top_p, repetition_penalty)
    context = model.embed.context  # earlier tokens the n-gram embedding of the next one needs
    out = torch.empty(input_ids.shape[0], prompt_len + max_new_tokens, dtype=input_ids.dtype,
                      device=input_ids.device)
    out[:, :prompt_len] = input_ids
    state, logits = model(input_ids, use_cache=True, keep_last=1, head=_head_last)
    finished = torch.zeros(input_ids.shape[0], dtype=torch.bool, device=input_ids.device)
    length = prompt_len
    for _ in range(max_new_tokens):
        token = params.pick(logits, out[:, prompt_len:length])
        if eos_token_id is not None:
            token = token.masked_fill(finished, eos_token_id)
            finished |= token == eos_token_id
        out[:, length] = token
        length += 1
        if eos_token_id is not None and bool(finished.all()):
            break
        pos = torch.full((out.shape[0], 1), length - 1, dtype=torch.long, device=out.device)
        prefix = out[:, max(0, length - 1 - context):length - 1] if context else None
        state, logits = model(out[:, length - 1:length], position_ids=pos, cache=state.cache, use_cache=True,
                              prefix_ids=prefix, head=_head_last)
    return out[:, :length]
