"""Portable model directories: ``model.safetensors`` + ``model.yaml`` (+ tokenizer files).

The directory layout is an interface shared with the reference
(``src/myk_llm/model/io.py:23-61``): a model exported by either framework loads in the
other.  With tied embeddings the output head is the token embedding, so
``lm_head.weight`` is not written and is the only key a load may find missing.
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
TIED_KEY = "lm_head.weight"


class ModelDirectory:
    """One exported model on disk."""

    def __init__(self, path) -> None:
        self.path = Path(path)

    @property
    def weights(self) -> Path:
        return self.path / WEIGHTS_FILE

    @property
    def config_file(self) -> Path:
        return self.path / CONFIG_FILE

    def write(self, config: ModelConfig, tensors: dict[str, torch.Tensor], tokenizer: str | None = None) -> None:
        self.path.mkdir(parents=True, exist_ok=True)
        host = {name: t.detach().cpu().contiguous() for name, t in tensors.items()
                if not (config.tie_embeddings and name == TIED_KEY)}
        save_file(host, str(self.weights))
        self.config_file.write_text(yaml.safe_dump(to_dict(config), sort_keys=False), encoding="utf-8")
        if tokenizer:
            from transformers import AutoTokenizer

            AutoTokenizer.from_pretrained(tokenizer).save_pretrained(str(self.path))

    def config(self) -> ModelConfig:
        return from_dict(ModelConfig, yaml.safe_load(self.config_file.read_text(encoding="utf-8")))

    def tensors(self) -> dict[str, torch.Tensor]:
        return load_file(str(self.weights))

    def instantiate(self, device="cuda", max_seq_len: int | None = None) -> MykLLM:
        cfg = self.config()
        if max_seq_len is not None:
            cfg.max_seq_len = max_seq_len
        model = MykLLM(cfg).to(device)
        result = model.load_state_dict(self.tensors(), strict=False)
        missing = set(result.missing_keys) - ({TIED_KEY} if cfg.tie_embeddings else set())
        if missing or result.unexpected_keys:
            raise KeyError(f"weight mismatch loading {self.path}: missing={sorted(missing)} "
                           f"unexpected={result.unexpected_keys}")
        return model.eval()


def save_model(directory, config: ModelConfig, state_dict: dict[str, torch.Tensor], tokenizer: str | None = None):
    ModelDirectory(directory).write(config, state_dict, tokenizer)


def load_model_config(directory) -> ModelConfig:
    return ModelDirectory(directory).config()


def load_state_dict(directory) -> dict[str, torch.Tensor]:
    return ModelDirectory(directory).tensors()


def load_model(directory, device="cuda", max_seq_len: int | None = None) -> MykLLM:
    return ModelDirectory(directory).instantiate(device, max_seq_len)
