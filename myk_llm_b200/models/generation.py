"""Autoregressive sampling with per-layer caches (the simple eager loop).

Same contract as the reference's ``generate`` (``src/myk_llm/model/generation.py:16-84``):
prefill with ``keep_last=1`` and the output head run as a forward head, then one token at
a time; greedy when ``temperature <= 0``, otherwise temperature / top-k / top-p sampling,
a CTRL repetition penalty over generated tokens only, rows padded with EOS once finished.

The fast path for serving (static caches, CUDA graphs, MTP speculative decoding) is
:mod:`myk_llm_b200.infer`.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .transformer import ModelOutput, MykLLM


def _last_logits(model: MykLLM, output: ModelOutput):
    return output, model.logits(output.hidden[:, -1]).float()


@torch.no_grad()
def generate(model: MykLLM, input_ids: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
             top_k: int | None = None, top_p: float | None = None, repetition_penalty: float = 1.0,
             eos_token_id: int | None = None) -> torch.Tensor:
    if input_ids.dim() != 2 or input_ids.size(1) == 0:
        raise ValueError("input_ids must be a non-empty (batch, seq_len) tensor")
    limit = model.config.max_seq_len
    if input_ids.size(1) + max_new_tokens > limit:
        raise ValueError(f"prompt ({input_ids.size(1)}) + max_new_tokens ({max_new_tokens}) exceeds max_seq_len {limit}")
    tokens = input_ids
    bsz = tokens.size(0)
    ctx = model.embed.context
    out, logits = model(tokens, use_cache=True, keep_last=1, head=_last_logits)
    cache = out.cache
    done = torch.zeros(bsz, dtype=torch.bool, device=tokens.device)
    plen = tokens.size(1)
    for _ in range(max_new_tokens):
        if repetition_penalty != 1.0 and tokens.size(1) > plen:
            seen = tokens[:, plen:]
            sc = logits.gather(1, seen)
            sc = torch.where(sc < 0, sc * repetition_penalty, sc / repetition_penalty)
            logits = logits.scatter(1, seen, sc)
        nxt = sample(logits, temperature, top_k, top_p)
        if eos_token_id is not None:
            nxt = torch.where(done, torch.full_like(nxt, eos_token_id), nxt)
            done |= nxt == eos_token_id
        tokens = torch.cat([tokens, nxt[:, None]], dim=1)
        if eos_token_id is not None and bool(done.all()):
            break
        pos = torch.full((bsz, 1), tokens.size(1) - 1, device=tokens.device, dtype=torch.long)
        prefix = tokens[:, -1 - ctx:-1] if ctx else None
        out, logits = model(tokens[:, -1:], position_ids=pos, cache=cache, use_cache=True, prefix_ids=prefix,
                            head=_last_logits)
        cache = out.cache
    return tokens


def sample(logits: torch.Tensor, temperature: float, top_k: int | None, top_p: float | None) -> torch.Tensor:
    if temperature <= 0.0:
        return logits.argmax(dim=-1)
    logits = logits / temperature
    if top_k is not None and top_k < logits.size(-1):
        cut = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < cut, float("-inf"))
    if top_p is not None and top_p < 1.0:
        srt, order = torch.sort(logits, descending=True, dim=-1)
        probs = F.softmax(srt, dim=-1)
        drop = probs.cumsum(-1) - probs > top_p
        srt = srt.masked_fill(drop, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter(1, order, srt)
    return torch.multinomial(F.softmax(logits, dim=-1), num_samples=1).squeeze(1)
