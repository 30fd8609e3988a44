"""Shared fixtures.  GPU tests carry ``@pytest.mark.gpu`` and need a B200 plus the built
extension; everything else runs on CPU."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running test")


def tiny_model_config(**overrides):
    """The reference's tiny test model (vocab 512, hidden 128, 4 layers GL, 2/1 heads of 64,
    window 64, DeltaNet 2x64, FFN x2), built through the typed override path."""
    from myk_llm_b200.configuration import apply_overrides, from_dict
    from myk_llm_b200.models import ModelConfig

    base = {
        "vocab_size": 512, "hidden_size": 128, "num_layers": 4, "layer_pattern": "GL", "max_seq_len": 256,
        "attention": {"num_heads": 2, "num_kv_heads": 1, "head_dim": 64, "sliding_window": 64},
        "deltanet": {"num_heads": 2, "head_dim": 64},
        "ffn": {"multiplier": 2.0, "multiple_of": 64},
    }
    return from_dict(ModelConfig, apply_overrides(base, [f"{k}={v}" for k, v in overrides.items()]))


@pytest.fixture
def tiny_config():
    return tiny_model_config


def cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False
