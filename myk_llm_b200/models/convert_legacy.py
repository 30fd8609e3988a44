"""Convert a pre-0.2 training checkpoint (one ``.pt`` holding ``model_config``,
``model_state_dict`` and ``training_args``) to the portable ``model.safetensors`` +
``model.yaml`` directory that :func:`myk_llm_b200.models.load_model` reads::

    python -m myk_llm_b200.models.convert_legacy checkpoints/200M-v5-sft/last.pt out/200M-v5-sft

The mapping is the reference's (``scripts/convert_legacy_checkpoint.py:17-63``), so
old checkpoints of either project load the same way:

* layer kinds: ``attn_types`` (full / sliding-window per layer) or a period
  ``full_attn_period`` (one global layer then ``period - 1`` local ones);
* old RoPE rule: the first layer and the sliding-window layers only
  (``global_rope: first`` when layer 0 is global);
* parameter names: ``token_embedding`` -> ``embed.token``, ``layers.N.attn_norm`` ->
  ``layers.N.mixer_norm``, ``layers.N.attn`` -> ``layers.N.mixer``.
"""

from __future__ import annotations

import argparse
import re

import torch

from .config import AttentionConfig, FFNConfig, ModelConfig
from .io import save_model

KIND_CODES = {"full_attention": "G", "sliding_window_attention": "L"}

NAME_MAP = (
    (re.compile(r"^token_embedding\."), "embed.token."),
    (re.compile(r"^layers\.(\d+)\.attn_norm\."), r"layers.\1.mixer_norm."),
    (re.compile(r"^layers\.(\d+)\.attn\."), r"layers.\1.mixer."),
)


def legacy_pattern(old: dict) -> str:
    kinds = old.get("attn_types")
    if kinds:
        return "".join(KIND_CODES[k] for k in kinds)
    return "G" + "L" * (old.get("full_attn_period", 4) - 1)


def convert_config(old: dict) -> ModelConfig:
    if old.get("dropout", 0.0):
        raise ValueError("legacy checkpoints trained with dropout are not supported")
    pattern = legacy_pattern(old)
    heads, hd = old["num_attention_heads"], old["head_dim"]
    return ModelConfig(
        vocab_size=old["vocab_size"], hidden_size=heads * hd, num_layers=old["num_layers"], layer_pattern=pattern,
        max_seq_len=old["max_seq_len"], tie_embeddings=old.get("tie_embeddings", True),
        initializer_range=old.get("initializer_range", 0.02),
        attention=AttentionConfig(num_heads=heads, num_kv_heads=old["num_kv_heads"], head_dim=hd,
                                  sliding_window=old["sliding_window_size"],
                                  rope_theta_local=old.get("sliding_window_rope_theta", 10_000.0),
                                  rope_theta_global=old.get("full_attention_rope_theta", 1_000_000.0),
                                  global_rope="first" if pattern[0] == "G" else "none"),
        ffn=FFNConfig(multiplier=old.get("ffn_multiplier", 4.0), multiple_of=old.get("ffn_multiple_of", 256)))


def rename(name: str) -> str:
    for pat, rep in NAME_MAP:
        name = pat.sub(rep, name)
    return name


def convert_state_dict(old: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    return {rename(k): v for k, v in old.items()}


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("checkpoint")
    ap.add_argument("output_dir")
    ap.add_argument("--tokenizer", default=None, help="default: the tokenizer recorded in the checkpoint")
    args = ap.parse_args(argv)
    ck = torch.load(args.checkpoint, map_location="cpu", weights_only=False)
    cfg = convert_config(ck["model_config"])
    tok = args.tokenizer or ck.get("training_args", {}).get("tokenizer")
    save_model(args.output_dir, cfg, convert_state_dict(ck["model_state_dict"]), tok)
    print(f"wrote {args.output_dir} ({cfg.num_layers} layers, pattern {cfg.layer_pattern})")


if __name__ == "__main__":
    main()
