"""Chat (or plain continuation) with an exported model directory.

    python -m myk_llm_b200.chat runs/200m-sft/export
    python -m myk_llm_b200.chat runs/200m-pt/export --raw --prompt "Once upon a time"
    python -m myk_llm_b200.chat runs/200m-pt/export --raw --prompt "..." --speculative   # MTP + CUDA graph

The directory is a portable export (``model.safetensors``, ``model.yaml``, tokenizer files).
A ``ChatSession`` keeps the conversation: SFT models get the tokenizer's chat template over
the whole history, base models (``--raw``) a plain continuation of the last text.  When
prompt plus reply would pass ``max_seq_len`` the oldest tokens are dropped.
``--speculative`` decodes greedily through the static-cache MTP engine
(:class:`myk_llm_b200.infer.StaticDecoder`, CUDA graphs).  The command line and the
helper functions ``build_prompt_ids`` / ``generate_reply`` are the reference's interface
(``src/myk_llm/chat.py:19-86``).
"""

from __future__ import annotations

import argparse
from dataclasses import dataclass, field

import torch

from .models import MykLLM, generate
from .models.io import load_model

EXIT_COMMANDS = frozenset({"exit", "quit", ":q"})


def _turns(history: list[tuple[str, str]], user_text: str) -> list[dict[str, str]]:
    msgs = [m for u, a in history for m in ({"role": "user", "content": u}, {"role": "assistant", "content": a})]
    return msgs + [{"role": "user", "content": user_text}]


def build_prompt_ids(model: MykLLM, tokenizer, history: list[tuple[str, str]], user_text: str,
                     raw: bool) -> torch.Tensor:
    """(1, n) token ids of the next turn on the model's device."""
    if raw:
        ids = tokenizer(user_text, add_special_tokens=False, return_tensors="pt")["input_ids"]
    else:
        ids = tokenizer.apply_chat_template(_turns(history, user_text), add_generation_prompt=True,
                                            return_tensors="pt", return_dict=True)["input_ids"]
    return ids.to(model.device)


def generate_reply(model: MykLLM, tokenizer, prompt_ids: torch.Tensor, max_tokens: int, speculative: bool = False,
                   **sampling) -> tuple[str, list[int], bool]:
    """(reply text, reply ids up to the end-of-turn token, whether that token came)."""
    budget = model.config.max_seq_len - max_tokens
    prompt_ids = prompt_ids[:, -budget:]  # drop the oldest context
    eos = tokenizer.eos_token_id
    if speculative:
        from .infer import StaticDecoder

        engine = StaticDecoder(model, batch_size=1, max_len=prompt_ids.shape[1] + max_tokens + 8)
        tokens, _ = engine.generate(prompt_ids, max_tokens)
    else:
        tokens = generate(model, prompt_ids, max_tokens, eos_token_id=eos, **sampling)
    reply = tokens[0, prompt_ids.shape[1]:].tolist()
    stopped = eos is not None and eos in reply
    if stopped:
        reply = reply[:reply.index(eos)]
    return tokenizer.decode(reply, skip_special_tokens=True).strip(), reply, stopped


@dataclass
class ChatSession:
    model: MykLLM
    tokenizer: object
    raw: bool = False
    max_tokens: int = 256
    speculative: bool = False
    sampling: dict = field(default_factory=dict)
    history: list[tuple[str, str]] = field(default_factory=list)

    @torch.no_grad()
    def say(self, text: str) -> str:
        ids = build_prompt_ids(self.model, self.tokenizer, [] if self.raw else self.history, text, self.raw)
        reply, _, _ = generate_reply(self.model, self.tokenizer, ids, self.max_tokens, self.speculative,
                                     **self.sampling)
        self.history.append((text, reply))
        return reply


def _repl(session: ChatSession) -> None:
    print("Type 'exit' to quit.")
    while True:
        try:
            text = input("user> ").strip()
        except EOFError:
            return
        if text.lower() in EXIT_COMMANDS:
            return
        if text:
            print(f"assistant> {session.say(text)}")


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

    session = ChatSession(load_model(args.model, device=args.device).eval(), AutoTokenizer.from_pretrained(args.model),
                          raw=args.raw, max_tokens=args.max_tokens, speculative=args.speculative,
                          sampling=dict(temperature=args.temperature, top_k=args.top_k, top_p=args.top_p,
                                        repetition_penalty=args.repetition_penalty))
    if args.prompt:
        print(session.say(args.prompt))
    else:
        _repl(session)


if __name__ == "__main__":
    main()
