"""Portable model directory: ``model.safetensors`` + ``model.yaml`` (+ tokenizer files).

The layout is the reference's (``src/myk_llm/model/io.py:23-61``) so exported models
load on either side: the tied ``lm_head.weight`` is dropped when embeddings are tied, and
loading is non-strict only for that key.
"""

from __future__ import annotations

from pathlib import Path

import torch
import yaml
from safetensors.torch import load_file, save_file

from ..configuration import from_dict, to_dict
from .config import ModelConfig
from .transformer import MykLLM

WEIGHTS_FILE = "model.safetensors"
CONFIG_FILE = "model.yaml"


def save_model(directory, config: ModelConfig, state_dict: dict[str, torch.Tensor], tokenizer: str | None = None):
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    tensors = {k: t.detach().to("cpu").contiguous() for k, t in state_dict.items()}
    if config.tie_embeddings:
        tensors.pop("lm_head.weight", None)
    save_file(tensors, str(directory / WEIGHTS_FILE))
    (directory / CONFIG_FILE).write_text(yaml.safe_dump(to_dict(config), sort_keys=False), encoding="utf-8")
    if tokenizer:
        from transformers import AutoTokenizer

        AutoTokenizer.from_pretrained(tokenizer).save_pretrained(str(directory))


def load_model_config(directory) -> ModelConfig:
    tree = yaml.safe_load((Path(directory) / CONFIG_FILE).read_text(encoding="utf-8"))
    return from_dict(ModelConfig, tree)


def load_state_dict(directory) -> dict[str, torch.Tensor]:
    return load_file(str(Path(directory) / WEIGHTS_FILE))


def load_model(directory, device="cuda", max_seq_len: int | None = None) -> MykLLM:
    config = load_model_config(directory)
    if max_seq_len is not None:
        config.max_seq_len = max_seq_len
    model = MykLLM(config).to(device)
    missing, unexpected = model.load_state_dict(load_state_dict(directory), strict=False)
    missing = [k for k in missing if not (config.tie_embeddings and k == "lm_head.weight")]
    if missing or unexpected:
        raise KeyError(f"weight mismatch loading {directory}: missing={missing} unexpected={unexpected}")
    return model.eval()
