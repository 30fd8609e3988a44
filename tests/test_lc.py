"""Long-context retrieval testbed: example construction (answers resolve through the
records), packing and targets, teacher-forced scoring, a short CPU run, early-exit
traces of a looped model, and the sweep tables."""

import json

import numpy as np
import pytest
import torch

from myk_llm_b200.configuration import apply_overrides, from_dict
from myk_llm_b200.data.config import IGNORE_INDEX
from myk_llm_b200.lc.data import PackedRetrieval, answer_targets
from myk_llm_b200.lc.eval import evaluate, score_batch
from myk_llm_b200.lc.halting import exit_iterations, tables, trace
from myk_llm_b200.lc.sweep import effective_length, report
from myk_llm_b200.lc.tasks import (EOS, KEY_BASE, NOISE_BASE, QUERY, VALUE_BASE, VOCAB_SIZE, TaskConfig,
                                   make_copy_example, make_example, resolve)
from myk_llm_b200.models import MykLLM


@pytest.mark.parametrize("hops", [[1], [1, 2, 3]])
@pytest.mark.parametrize("cot", [False, True])
def test_answers_resolve_through_the_records(hops, cot):
    task = TaskConfig(num_records=6, num_queries=3, hops=hops, cot=cot)
    rng = np.random.default_rng(0)
    for _ in range(20):
        ex = make_example(rng, task, 512)
        assert len(ex.ids) == 512 and len(ex.answers) == 3
        for (s, e), h in zip(ex.answers, ex.hops):
            assert ex.ids[e - 1] == EOS
            q = s - 1 - task.key_len
            assert ex.ids[q] == QUERY
            key = ex.ids[q + 1:s].tolist()
            value = resolve(ex.ids, key, task.key_len)
            assert ex.ids[e - 1 - task.value_len:e - 1].tolist() == value
            assert (e - s - 1) == task.value_len + (task.key_len * (h - 1) if cot else 0)
        assert np.all(ex.ids[: ex.answers[0][0]] < VOCAB_SIZE)
        assert 0.0 <= min(ex.depths) and max(ex.depths) < 1.0


def test_alphabets_are_disjoint_and_scaling():
    task = TaskConfig(num_records=16, num_queries=4, scale_records=True, max_len=1024)
    assert task.records_at(512) == 8 and task.records_at(2048) == 32
    ex = make_example(np.random.default_rng(1), task, 1024)
    ctx = ex.ids[: ex.answers[0][0]]
    assert np.all((ctx < 4) | ((ctx >= KEY_BASE) & (ctx < VOCAB_SIZE)))
    assert np.any(ctx >= NOISE_BASE) and np.any((ctx >= VALUE_BASE) & (ctx < NOISE_BASE))


def test_copy_examples_and_targets():
    task = TaskConfig(copy_fraction=1.0, copy_min=8, copy_max=8, max_len=256)
    ex = make_copy_example(np.random.default_rng(0), task)
    assert len(ex.ids) == 16 and np.array_equal(ex.ids[:8], ex.ids[8:])
    tg = answer_targets(ex)
    assert np.all(tg[:8] == IGNORE_INDEX) and np.array_equal(tg[8:15], ex.ids[9:16]) and tg[15] == IGNORE_INDEX


def test_packed_rows():
    task = TaskConfig(min_len=64, max_len=256, num_records=2, num_queries=1, copy_fraction=0.3, copy_min=4,
                      copy_max=16, min_records=1)
    b = next(iter(PackedRetrieval(task, batch_rows=3, seed=0)))
    assert b.input_ids.shape == (3, 256)
    assert all(int(l.sum()) == 256 for l in b.seqlens)
    assert (b.targets != IGNORE_INDEX).any()


def _tiny(loop: bool = False):
    ov = ["vocab_size=512", "hidden_size=64", "num_layers=4", "layer_pattern=G", "max_seq_len=1024",
          "attention.num_heads=2", "attention.num_kv_heads=2", "attention.head_dim=32"]
    if loop:
        ov += ["loop.core=2", "loop.prelude=2", "loop.iterations=2"]
    from myk_llm_b200.models import ModelConfig

    torch.manual_seed(0)
    return MykLLM(from_dict(ModelConfig, apply_overrides({}, ov))).eval()


def test_teacher_forced_scoring_matches_its_definition():
    model = _tiny()
    task = TaskConfig(num_records=2, num_queries=2, max_len=256)
    exs = [make_example(np.random.default_rng(k), task, 256) for k in range(2)]
    got = score_batch(model, exs)
    with torch.no_grad():
        for r, ex in enumerate(exs):
            ids = torch.from_numpy(ex.ids)[None]
            pred = model.logits(model(ids).hidden)[0].argmax(-1)
            for (s, e), g in zip(ex.answers, got[2 * r:2 * r + 2]):
                assert g == bool(torch.equal(pred[s - 1:e - 1], ids[0, s:e]))
    res = evaluate(model, task, [128, 256], queries=4, seed=0)
    assert set(res["accuracy"]) == {128, 256} and len(res["depth"][256]) == task.depth_buckets


def test_training_run_writes_results(tmp_path):
    from myk_llm_b200.lc.train import LcConfig, train

    ov = ["model.vocab_size=512", "model.hidden_size=64", "model.num_layers=2", "model.layer_pattern=G",
          "model.max_seq_len=512", "model.attention.num_heads=2", "model.attention.num_kv_heads=2",
          "model.attention.head_dim=32", "steps=3", "batch_rows=2", "num_workers=0", "log_interval=1",
          "eval_interval=2", "eval_queries=4", "final_eval_queries=4", "task.min_len=64", "task.max_len=256",
          "task.num_records=2", "task.num_queries=1", "task.eval_lengths=[128,512]", "task.eval_hops=[1,2]",
          "optimizer.name=adamw", f"output_dir={tmp_path}"]
    cfg = from_dict(LcConfig, apply_overrides({}, ov))
    train(cfg, device="cpu")
    res = json.loads((tmp_path / "lc" / "results.json").read_text())
    assert set(res["accuracy"]) == {"128", "512"} and res["train_len"] == 256
    assert res["scan"] and set(res["scan"][0]["hops"]["512"]) <= {"1", "2"}


def test_halting_trace_and_rules():
    model = _tiny(loop=True)
    task = TaskConfig(num_records=2, num_queries=2, max_len=256, hops=[1, 2])
    exs = [make_example(np.random.default_rng(k), task, 256) for k in range(2)]
    tr = trace(model, exs, iterations=3)
    assert tr["correct"].shape == (4, 3) and np.isinf(tr["delta"][:, 0]).all()
    sig = np.array([[np.inf, 0.5, 0.01], [np.inf, 0.001, 0.0]])
    assert exit_iterations(sig, "<", 0.1, 3).tolist() == [3, 2]
    data = {**tr, "hops": np.array([h for e in exs for h in e.hops])}
    assert any("Exit rules" in line for line in tables("x", data, budget=3))


def test_sweep_tables(tmp_path):
    assert effective_length({"512": 1.0, "1024": 0.95, "2048": 0.4}, 0.9) == 1024
    for name, acc in [("needle-g-s0", {"512": 1.0, "1024": 0.8}), ("needle-g-s1", {"512": 1.0, "1024": 1.0})]:
        d = tmp_path / name
        d.mkdir()
        (d / "results.json").write_text(json.dumps({
            "run_name": name, "accuracy": acc, "train_len": 512, "train_minutes": 2.0,
            "depth": {"1024": [1.0, 0.5]}, "hops": {"1024": {"1": 0.9}}, "scan": []}))
    table = report(tmp_path, at=1024)
    assert "| needle-g | 2 |" in table and "needle depth" in table
