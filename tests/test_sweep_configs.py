"""Every committed sweep file expands into runs whose configs load with this framework's
schema (base file + the run's overrides), so a sweep shared with the reference runs here
unchanged."""

from pathlib import Path

import pytest
import yaml

from myk_llm_b200.configuration import load_config
from myk_llm_b200.utils.sweep import plan

ROOT = Path(__file__).resolve().parents[1]
SWEEPS = sorted((ROOT / "configs").glob("*/sweeps/*.yaml"))


def _schema(kind: str):
    if kind == "lc":
        from myk_llm_b200.lc.train import LcConfig
        return LcConfig
    if kind == "arith":
        from myk_llm_b200.arith.train import ArithConfig
        return ArithConfig
    from myk_llm_b200.train.config import TrainConfig
    return TrainConfig


@pytest.mark.parametrize("path", SWEEPS, ids=[f"{p.parent.parent.name}/{p.name}" for p in SWEEPS])
def test_sweep_expands_to_loadable_configs(path, monkeypatch):
    monkeypatch.chdir(ROOT)
    spec = yaml.safe_load(path.read_text())
    runs = plan(spec)
    assert runs and len({name for name, _, _ in runs}) == len(runs)
    schema = _schema(path.parent.parent.name)
    for name, base, overrides in runs:
        load_config(schema, base, list(overrides) + [f"run_name={name}"])
