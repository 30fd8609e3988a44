from .config import (AttentionConfig, CrossDecoderConfig, DeltaNetConfig, FFNConfig, LoopConfig, ModelConfig,
                     MTPConfig, NgramEmbeddingConfig, ResidualConfig)
from .generation import generate
from .io import load_model, load_model_config, save_model
from .transformer import ModelOutput, MykLLM

__all__ = [
    "AttentionConfig", "CrossDecoderConfig", "DeltaNetConfig", "FFNConfig", "LoopConfig", "ModelConfig", "MTPConfig",
    "MykLLM", "ModelOutput", "NgramEmbeddingConfig", "ResidualConfig", "generate", "load_model", "load_model_config",
    "save_model",
]
