"""Arithmetic testbed: formats round-trip, supervision mask, packing, digit indices, a
short CPU training run end to end, and sweep planning / reporting."""

import json
import random

import pytest
import torch

from myk_llm_b200.arith.data import PackedArithmetic, encode_example
from myk_llm_b200.arith.model import ArithModel, DigitEmbeddingConfig, digit_indices, evaluate_lengths
from myk_llm_b200.arith.sweep import extra_digits, report
from myk_llm_b200.arith.tasks import (CharTokenizer, TaskConfig, add_fillers, parse_answer, render, sample_problem,
                                      true_answer)
from myk_llm_b200.configuration import apply_overrides, from_dict
from myk_llm_b200.data.config import IGNORE_INDEX
from myk_llm_b200.utils.sweep import plan


@pytest.mark.parametrize("op", ["add", "mul"])
@pytest.mark.parametrize("fmt", ["direct", "reverse", "cot"])
@pytest.mark.parametrize("rev", [False, True])
def test_answers_parse_back(op, fmt, rev):
    task = TaskConfig(op=op, format=fmt, train_digits=6, reverse_operands=rev)
    rng = random.Random(1)
    for _ in range(300):
        a, b = sample_problem(rng, task)
        p, c = render(a, b, task)
        assert p.endswith("=") and c.endswith("$")
        assert parse_answer(c, task) == true_answer(a, b, task)


def test_chain_of_thought_strings():
    assert render(123, 456, TaskConfig(op="add"))[1] == "3+6+0:09,2+5+0:07,1+4+0:05|579$"
    assert render(99, 1, TaskConfig(op="add"))[1] == "9+1+0:10,9+0+1:10|100$"
    assert render(37, 24, TaskConfig(op="mul"))[1] == "841;047>888|888$"
    assert render(123, 45, TaskConfig(op="add", format="reverse", reverse_operands=True)) == ("321+54=", "861$")


def test_fillers_keep_the_problem():
    rng = random.Random(0)
    p = add_fillers("123+45=", rng, 1.0, 2)
    assert p.replace("_", "") == "123+45=" and p.endswith("=") and p[0] == "1" and "_" in p


def test_only_the_completion_is_supervised():
    tok = CharTokenizer()
    ids, tg = encode_example(tok, "12+3=", "15$")
    assert tok.decode(ids) == "12+3=15$"
    assert [tok.decode([t]) for t in tg if t != IGNORE_INDEX] == ["1", "5", "$"]
    assert tg[-1] == IGNORE_INDEX and tg[3] == IGNORE_INDEX


def test_rows_are_full_and_segmented():
    b = next(iter(PackedArithmetic(TaskConfig(train_digits=4), batch_rows=3, row_len=128, seed=0)))
    assert b.input_ids.shape == (3, 128)
    for lens in b.seqlens:
        assert int(lens.sum()) == 128


def test_digit_indices_restart_per_number():
    tok = CharTokenizer()
    ids = torch.tensor([tok.encode("123+45=5")])
    assert digit_indices(ids, torch.tensor(tok.digit_ids)).tolist() == [[1, 2, 3, 0, 1, 2, 0, 1]]


def _tiny_config(tmp_path, **extra):
    from myk_llm_b200.arith.train import ArithConfig

    ov = ["model.vocab_size=32", "model.hidden_size=64", "model.num_layers=2", "model.layer_pattern=G",
          "model.max_seq_len=256", "model.attention.num_heads=2", "model.attention.num_kv_heads=2",
          "model.attention.head_dim=32", "steps=4", "batch_rows=2", "row_len=128", "num_workers=0",
          "log_interval=2", "eval_interval=2", "eval_examples=4", "final_eval_examples=4",
          "task.train_digits=3", "task.eval_digits=[1,2,4]", "optimizer.name=adamw", f"output_dir={tmp_path}"]
    ov += [f"{k}={v}" for k, v in extra.items()]
    return from_dict(ArithConfig, apply_overrides({}, ov))


@pytest.mark.parametrize("abacus", [False, True])
def test_training_run_writes_results(tmp_path, abacus):
    from myk_llm_b200.arith.train import train

    cfg = _tiny_config(tmp_path, **{"digit_embedding.enabled": str(abacus).lower()})
    res = train(cfg, device="cpu")
    out = json.loads((tmp_path / "arith" / "results.json").read_text())
    assert set(out["accuracy"]) == {"1", "2", "4"} and 0.0 <= res["in_distribution"] <= 1.0
    assert (tmp_path / "arith" / "model.pt").exists()


def test_greedy_stays_in_the_character_set():
    from conftest import tiny_model_config

    torch.manual_seed(0)
    model = ArithModel(tiny_model_config(vocab_size=64), DigitEmbeddingConfig()).eval()
    outs = model.greedy_complete(["12+34=", "5+6="], 6)
    assert all(set(o) <= set(CharTokenizer().chars) for o in outs)
    acc = evaluate_lengths(model, TaskConfig(format="direct", train_digits=2), [1, 2], examples=3, seed=0)
    assert set(acc) == {1, 2}


def test_sweep_plan_and_report(tmp_path):
    runs = plan({"configs": {"add": "a.yaml"}, "axes": {"fmt": {"cot": ["task.format=cot"], "direct": []},
                                                       "seed": {"s0": ["seed=0"], "s1": ["seed=1"]}},
                 "overrides": ["steps=10"]})
    assert [r[0] for r in runs] == ["add-cot-s0", "add-cot-s1", "add-direct-s0", "add-direct-s1"]
    assert runs[0][2] == ["steps=10", "task.format=cot", "seed=0"]
    for name, acc in [("add-cot-s0", {"1": 1.0, "2": 1.0, "3": 0.6, "4": 0.2}),
                      ("add-cot-s1", {"1": 1.0, "2": 1.0, "3": 0.8, "4": 0.6})]:
        d = tmp_path / name
        d.mkdir()
        (d / "results.json").write_text(json.dumps({"run_name": name, "accuracy": acc, "train_digits": 2,
                                                    "train_minutes": 1.0}))
    assert extra_digits({"train_digits": 2, "accuracy": {"3": 0.6, "4": 0.2}}) == 1
    table = report(tmp_path)
    assert "| add-cot | 2 |" in table and "1.5" in table
