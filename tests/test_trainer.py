"""Trainer on CPU (the tiny dense correctness config): steps run, loss falls, DCP checkpoints resume
bit-exactly, incomplete checkpoints are ignored, and the portable export loads."""

import json
import shutil

import pytest
import torch

from myk_llm_b200.configuration import load_config
from myk_llm_b200.parallel.distributed import DistInfo
from myk_llm_b200.train.config import TrainConfig
from myk_llm_b200.train.trainer import Trainer


def _cfg(tmp_path, **ov):
    ovs = [f"output_dir={tmp_path}", "steps=6", "logging.interval=2", "model.num_layers=2",
           "data.seq_len=64", "data.micro_batch_size=2", "global_batch_size=4", "model.max_seq_len=64"]
    ovs += [f"{k}={v}" for k, v in ov.items()]
    return load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", ovs)


CPU = DistInfo(0, 1, 0, torch.device("cpu"))


def test_train_steps_reduce_loss(tmp_path):
    cfg = _cfg(tmp_path, steps=30, **{"optimizer.lr": 3e-3, "data.synthetic.mean_doc_len": 1000})
    tr = Trainer(cfg, CPU)
    batches = [tr.loader.next_batch() for _ in range(2)]
    losses = [float(tr.train_step(batches, s)["loss"]) for s in range(1, 31)]
    assert losses[-1] < losses[0] - 0.5, losses


def test_resume_is_exact(tmp_path):
    cfg = _cfg(tmp_path, **{"checkpoint.interval": 3, "checkpoint.final": True})
    Trainer(cfg, CPU).fit("none")
    run = tmp_path / cfg.run_name
    final = Trainer(cfg, CPU)
    from myk_llm_b200.train.checkpoint import latest_checkpoint, load_checkpoint

    ck = latest_checkpoint(run)
    assert ck.name == "step_0000006"
    # re-run steps 4..6 from the step-3 checkpoint and compare with the step-6 weights
    shutil.rmtree(ck)
    t2 = Trainer(cfg, CPU)
    t2.fit("auto")
    ref = Trainer(cfg, CPU)
    load_checkpoint(latest_checkpoint(run), ref.model, ref.optimizers, CPU)
    a = dict(t2.model.named_parameters())
    for n, p in ref.model.named_parameters():
        assert torch.equal(p, a[n]), n


def test_incomplete_checkpoint_ignored(tmp_path):
    from myk_llm_b200.train.checkpoint import latest_checkpoint

    cfg = _cfg(tmp_path, **{"checkpoint.interval": 3, "checkpoint.final": True})
    Trainer(cfg, CPU).fit("none")
    run = tmp_path / cfg.run_name
    (run / "checkpoints" / "step_0000009").mkdir(parents=True)
    assert latest_checkpoint(run).name == "step_0000006"


def test_export_loads(tmp_path):
    from myk_llm_b200.models import load_model

    cfg = _cfg(tmp_path, **{"checkpoint.interval": 6, "checkpoint.final": True})
    Trainer(cfg, CPU).fit("none")
    d = tmp_path / cfg.run_name / "checkpoints" / "step_0000006"
    m = load_model(d, device="cpu")
    assert (d / "model.safetensors").exists() and (d / "trainer.json").exists()
    assert json.loads((d / "trainer.json").read_text())["step"] == 6
    assert m.config.hidden_size == 256


def test_non_finite_loss_stops_the_run(tmp_path):
    """A non-finite loss or gradient norm is caught at the next logging sync."""
    cfg = _cfg(tmp_path)
    tr = Trainer(cfg, CPU)
    with torch.no_grad():
        next(tr.model.parameters()).fill_(float("nan"))
    with pytest.raises(FloatingPointError, match="non-finite"):
        tr.fit("none")
