"""Chat or plain text completion with an exported model directory.

    python -m myk_llm_b200.chat runs/200m-sft/export
    python -m myk_llm_b200.chat runs/200m-pt/export --raw --prompt "Once upon a time"
    python -m myk_llm_b200.chat runs/200m-pt/export --raw --prompt "..." --speculative   # MTP + CUDA graph

The directory holds ``model.safetensors``, ``model.yaml`` and the tokenizer files
(:func:`myk_llm_b200.models.io.save_model`).  Turns use the tokenizer's chat template
(SFT models) or raw continuation (base models); the oldest context is dropped once the
prompt plus the reply would exceed ``max_seq_len``.  ``--speculative`` decodes greedily
through the static-cache MTP engine (:class:`myk_llm_b200.infer.StaticDecoder`).

Interface of the reference's ``src/myk_llm/chat.py:19-86``.
"""

from __future__ import annotations

import argparse

import torch

from .models import MykLLM, generate
from .models.io import load_model

EXIT_COMMANDS = {"exit", "quit", ":q"}


def build_prompt_ids(model: MykLLM, tokenizer, history: list[tuple[str, str]], user_text: str,
                     raw: bool) -> torch.Tensor:
    """Token ids of the next turn: chat template (with the history) or raw text."""
    if raw:
        ids = tokenizer(user_text, add_special_tokens=False, return_tensors="pt")["input_ids"]
    else:
        messages = []
        for u, a in history:
            messages.append({"role": "user", "content": u})
            messages.append({"role": "assistant", "content": a})
        messages.append({"role": "user", "content": user_text})
        ids = tokenizer.apply_chat_template(messages, add_generation_prompt=True, return_tensors="pt",
                                            return_dict=True)["input_ids"]
    return ids.to(next(model.parameters()).device)


def generate_reply(model: MykLLM, tokenizer, prompt_ids: torch.Tensor, max_tokens: int, speculative: bool = False,
                   **sampling) -> tuple[str, list[int], bool]:
    """(reply text, reply ids, whether the end-of-turn token was produced)."""
    keep = model.config.max_seq_len - max_tokens
    prompt_ids = prompt_ids[:, -keep:]
    eos = tokenizer.eos_token_id
    if speculative:
        from .infer import StaticDecoder

        dec = StaticDecoder(model, batch_size=1, max_len=prompt_ids.size(1) + max_tokens + 8)
        out, _ = dec.generate(prompt_ids, max_tokens)
    else:
        out = generate(model, prompt_ids, max_tokens, eos_token_id=eos, **sampling)
    ids = out[0, prompt_ids.size(1):].tolist()
    stopped = eos is not None and eos in ids
    if stopped:
        ids = ids[:ids.index(eos)]
    return tokenizer.decode(ids, skip_special_tokens=True).strip(), ids, stopped


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("model", help="exported model directory")
    ap.add_argument("--prompt", default="", help="answer one prompt and exit")
    ap.add_argument("--raw", action="store_true", help="plain continuation (base models)")
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--top-k", type=int, default=50)
    ap.add_argument("--top-p", type=float, default=0.95)
    ap.add_argument("--repetition-penalty", type=float, default=1.1)
    ap.add_argument("--speculative", action="store_true", help="greedy MTP speculative decoding (CUDA)")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    args = ap.parse_args(argv)

    from transformers import AutoTokenizer

    model = load_model(args.model, device=args.device).eval()
    tokenizer = AutoTokenizer.from_pretrained(args.model)
    sampling = dict(temperature=args.temperature, top_k=args.top_k, top_p=args.top_p,
                    repetition_penalty=args.repetition_penalty)
    with torch.no_grad():
        if args.prompt:
            ids = build_prompt_ids(model, tokenizer, [], args.prompt, args.raw)
            print(generate_reply(model, tokenizer, ids, args.max_tokens, args.speculative, **sampling)[0])
            return
        history: list[tuple[str, str]] = []
        print("Type 'exit' to quit.")
        while True:
            try:
                text = input("user> ").strip()
            except EOFError:
                break
            if not text:
                continue
            if text.lower() in EXIT_COMMANDS:
                break
            ids = build_prompt_ids(model, tokenizer, history, text, args.raw)
            reply, _, _ = generate_reply(model, tokenizer, ids, args.max_tokens, args.speculative, **sampling)
            print(f"assistant> {reply}")
            history.append((text, reply))


if __name__ == "__main__":
    main()
