"""DCP checkpoints interchange with the reference implementation, both directions (CPU):
a checkpoint written by the reference's own ``save_checkpoint`` (model + Muon / AdamW state
after one step) loads into this framework's model and optimizers with identical values,
and one written here loads into the reference.  Runs against the reference package
installed under ``baseline/_ref``; skipped where it is not installed."""

import importlib
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

MODEL = {"vocab_size": 512, "hidden_size": 128, "num_layers": 2, "layer_pattern": "GL", "max_seq_len": 128,
         "tie_embeddings": False,
         "attention": {"num_heads": 2, "num_kv_heads": 1, "head_dim": 64, "sliding_window": 64},
         "ffn": {"multiplier": 2.0, "multiple_of": 64},
         "ngram": {"orders": [2, 3], "num_buckets": 256, "dim": 32},
         "mtp": {"depth": 1}}
OPT = {"name": "muon", "lr": 1e-3}


def _ref():
    if not (REF / "myk_llm" / "__init__.py").exists():
        pytest.skip("reference not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    try:
        return {m: importlib.import_module(f"myk_llm.{m}") for m in
                ("configuration", "model", "train.config", "train.optim", "train.checkpoint", "train.distributed")}
    except Exception as err:  # an optional dependency of the reference is missing here
        pytest.skip(f"reference does not import: {err}")


def _build(cfg_mod, model_mod, train_cfg_mod, optim_mod, seed):
    torch.manual_seed(seed)
    mcfg = cfg_mod.from_dict(model_mod.ModelConfig, MODEL)
    model = model_mod.MykLLM(mcfg)
    opts = optim_mod.build_optimizers(model, cfg_mod.from_dict(train_cfg_mod.OptimizerConfig, OPT))
    for p in model.parameters():  # one step so that the optimizers have state
        p.grad = torch.randn_like(p) * 0.01
    for o in opts:
        o.step()
    return model, opts


def _ours():
    from myk_llm_b200 import configuration, models
    from myk_llm_b200.train import checkpoint, config, optim
    from myk_llm_b200.parallel import distributed
    return {"configuration": configuration, "model": models, "train.config": config, "train.optim": optim,
            "train.checkpoint": checkpoint, "train.distributed": distributed}


def _state(model, opts):
    from torch.distributed.checkpoint.state_dict import get_state_dict

    ms, os_ = get_state_dict(model, opts)
    return ms, os_


def _same(a, b):
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k].float(), b[k].float()), k


def _roundtrip(src, dst, tmp_path):
    model_s, opts_s = _build(src["configuration"], src["model"], src["train.config"], src["train.optim"], 0)
    info_s = src["train.distributed"].DistInfo(0, 1, 0, torch.device("cpu"))
    d = tmp_path / "step_0000001"
    src["train.checkpoint"].save_checkpoint(d, model_s, opts_s, {"step": 1, "tokens": 0, "world_size": 1}, {},
                                            info_s, False)
    model_d, opts_d = _build(dst["configuration"], dst["model"], dst["train.config"], dst["train.optim"], 1)
    info_d = dst["train.distributed"].DistInfo(0, 1, 0, torch.device("cpu"))
    dst["train.checkpoint"].load_checkpoint(d, model_d, opts_d, info_d)
    ms, os_ = _state(model_s, opts_s)
    md, od = _state(model_d, opts_d)
    _same(ms, md)
    assert os_["state"].keys() == od["state"].keys()
    for k in os_["state"]:
        sa, sb = os_["state"][k], od["state"][k]
        assert sa.keys() == sb.keys(), k
        for kk in sa:
            va, vb = sa[kk], sb[kk]
            if torch.is_tensor(va):
                assert torch.equal(va.float(), vb.float()), (k, kk)
            else:
                assert va == vb, (k, kk)


def test_reference_checkpoint_loads_here(tmp_path):
    _roundtrip(_ref(), _ours(), tmp_path)


def test_checkpoint_from_here_loads_in_reference(tmp_path):
    _roundtrip(_ours(), _ref(), tmp_path)
