"""Command-line tools beside the data / model / training packages, run on tiny local
inputs on CPU: corpus pretokenization into shards, SFT data building and tokenization,
tokenizer pruning, legacy checkpoint conversion, sweep summaries and the small helpers."""

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
WORDS = ("alpha beta gamma delta epsilon zeta eta theta iota kappa lambda mu nu xi omicron pi rho sigma tau "
         "upsilon phi chi psi omega").split()
SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def _text(rng, n):
    return " ".join(rng.choice(WORDS) for _ in range(n))


@pytest.fixture(scope="module")
def tok_dir(tmp_path_factory):
    """A byte-level BPE tokenizer trained on the test vocabulary (a few hundred tokens)."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    rng = np.random.default_rng(0)
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=400, special_tokens=SPECIALS,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator([_text(rng, 40) for _ in range(300)] + ["Hello, world! 123 user assistant system"], trainer)
    d = tmp_path_factory.mktemp("tok")
    tok.save(str(d / "tokenizer.json"))
    from transformers import PreTrainedTokenizerFast

    fast = PreTrainedTokenizerFast(tokenizer_object=tok, eos_token="<|endoftext|>")
    fast.chat_template = (ROOT / "assets" / "chatml_no_think.jinja").read_text()
    fast.save_pretrained(str(d))
    return d


def _corpus(tmp_path, docs=60):
    rng = np.random.default_rng(1)
    p = tmp_path / "corpus.jsonl"
    with p.open("w") as f:
        for i in range(docs):
            f.write(json.dumps({"text": f"{i} " + _text(rng, int(rng.integers(20, 80)))}) + "\n")
    return p


def test_pretokenize_local_corpus_into_shards(tmp_path, tok_dir):
    from tokenizers import Tokenizer

    from myk_llm_b200.data import pretokenize
    from myk_llm_b200.data.shards import ShardSource
    from myk_llm_b200.data.config import SourceConfig

    corpus = _corpus(tmp_path)
    out = tmp_path / "shards"
    pretokenize.main(["--path", str(corpus), "--tokenizer", str(tok_dir), "--target-tokens", "1e6",
                      "--val-fraction", "0.1", "--shard-tokens", "2000", "--shuffle-buffer", "0",
                      "--output", str(out)])
    tok = Tokenizer.from_file(str(tok_dir / "tokenizer.json"))
    eos = tok.token_to_id("<|endoftext|>")
    lines = [json.loads(line)["text"] for line in corpus.read_text().splitlines()]
    want = sum(len(tok.encode(t, add_special_tokens=False).ids) + 1 for t in lines)
    metas = {s: json.loads((out / s / "meta.json").read_text()) for s in ("train", "val")}
    assert metas["train"]["eos_id"] == eos
    assert metas["train"]["num_tokens"] + metas["val"]["num_tokens"] == want
    assert metas["val"]["num_tokens"] > 0 and len(metas["train"]["shards"]) >= 2
    src = ShardSource(SourceConfig(name="t", path=str(out / "train")), 64)
    row = src.window(0, document_masking=True)
    assert row["seqlens"].sum() == 64
    allt = np.concatenate([np.fromfile(out / "train" / sh["file"], dtype=np.uint32)
                           for sh in metas["train"]["shards"]])
    assert (allt == eos).sum() == sum(len(np.load(out / "train" / sh["file"].replace(".bin", ".docs.npy")))
                                       for sh in metas["train"]["shards"])


def test_build_sft_data_from_local_files_dedups_and_splits(tmp_path):
    from myk_llm_b200.data import build_sft_data

    rows = [{"messages": [{"role": "user", "content": f"question number {i} about things"},
                          {"role": "assistant", "content": f"an answer that is long enough {i}"}]} for i in range(50)]
    rows += rows[:10]  # duplicates
    rows.append({"conversations": [{"from": "human", "value": "a sharegpt style question here"},
                                   {"from": "gpt", "value": "and its sharegpt style answer"}]})
    rows.append({"messages": [{"role": "user", "content": "too short"}]})
    src = tmp_path / "raw.jsonl"
    src.write_text("\n".join(json.dumps(r) for r in rows))
    out = tmp_path / "sft"
    build_sft_data.main(["--out-dir", str(out), "--source", f"mine=local:{src}", "--val-frac", "0.1",
                         "--min-chars", "10"])
    train = [json.loads(x) for x in (out / "train.jsonl").read_text().splitlines()]
    val = [json.loads(x) for x in (out / "val.jsonl").read_text().splitlines()]
    assert len(train) + len(val) == 51 and len(val) == 5
    assert all(m["role"] in ("user", "assistant", "system") for r in train + val for m in r["messages"])


def test_tokenize_sft_masks_assistant_turns(tmp_path, tok_dir):
    from myk_llm_b200.data import tokenize_sft

    data = tmp_path / "chat.jsonl"
    data.write_text("\n".join(json.dumps({"messages": [{"role": "user", "content": "alpha beta"},
                                                       {"role": "assistant", "content": "gamma delta " * (i + 1)}]})
                              for i in range(4)))
    tokenize_sft.main(["--data", str(data), "--tokenizer", str(tok_dir), "--output", str(tmp_path / "out" / "train")])
    meta = json.loads((tmp_path / "out" / "train.meta.json").read_text())
    toks = np.fromfile(tmp_path / "out" / "train.tokens.bin", dtype=np.uint32)
    mask = np.fromfile(tmp_path / "out" / "train.loss_mask.bin", dtype=np.uint8)
    spans = np.load(tmp_path / "out" / "train.spans.npy")
    assert len(spans) == 4 and len(toks) == len(mask) == spans[-1][1]
    assert 0 < mask.sum() < len(mask)
    assert meta["num_tokens"] == len(toks)


def test_prune_tokenizer_keeps_encoding_closed(tmp_path, tok_dir):
    from tokenizers import Tokenizer

    from myk_llm_b200.data import prune_tokenizer

    corpus = tmp_path / "c.txt"
    rng = np.random.default_rng(3)
    corpus.write_text("\n".join(_text(rng, 30) for _ in range(200)))
    src = Tokenizer.from_file(str(tok_dir / "tokenizer.json"))
    target = 300
    prune_tokenizer.main(["--source", str(tok_dir), "--corpus", str(corpus), "--vocab-size", str(target),
                          "--output", str(tmp_path / "pruned")])
    new = Tokenizer.from_file(str(tmp_path / "pruned" / "tokenizer.json"))
    row_map = np.load(tmp_path / "pruned" / "embedding_row_map.npy")
    assert new.get_vocab_size() == len(row_map) <= target
    for text in ["alpha gamma omega", "Hello, world! 123", "unseen ž 漢字 text"]:
        ids = new.encode(text, add_special_tokens=False).ids
        assert new.decode(ids) == text
        # every new id maps back to the same string in the source vocabulary
        assert [src.id_to_token(int(row_map[i])) for i in ids] == [new.id_to_token(i) for i in ids]
    for s in SPECIALS:
        assert new.token_to_id(s) is not None
    report = json.loads((tmp_path / "pruned" / "prune_report.json").read_text())
    assert report["kept"] == len(row_map) and 0 < report["corpus_coverage_of_kept"] < 1
    # a larger budget keeps a superset, covering more of the corpus
    tj = json.loads((tok_dir / "tokenizer.json").read_text())
    counts = prune_tokenizer.count_frequencies(src, corpus.read_text().splitlines(), src.get_vocab_size())
    small, big = (prune_tokenizer.prune(tj, counts, n) for n in (280, 340))
    assert set(small[1].tolist()) <= set(big[1].tolist())
    assert big[2]["corpus_coverage_of_kept"] > small[2]["corpus_coverage_of_kept"]


def test_convert_legacy_checkpoint_round_trip(tmp_path):
    from conftest import tiny_model_config
    from myk_llm_b200.models import MykLLM, load_model
    from myk_llm_b200.models import convert_legacy

    old_cfg = {"vocab_size": 256, "num_attention_heads": 4, "head_dim": 16, "num_kv_heads": 2, "num_layers": 4,
               "attn_types": ["full_attention", "sliding_window_attention", "sliding_window_attention",
                              "full_attention"],
               "max_seq_len": 128, "sliding_window_size": 32, "ffn_multiplier": 2.0, "ffn_multiple_of": 32}
    cfg = convert_legacy.convert_config(old_cfg)
    assert cfg.layer_pattern == "GLLG" and cfg.hidden_size == 64 and cfg.attention.global_rope == "first"
    assert convert_legacy.legacy_pattern({"full_attn_period": 3}) == "GLL"
    torch.manual_seed(0)
    model = MykLLM(cfg)
    legacy = {}
    for k, v in model.state_dict().items():
        k = k.replace("embed.token.", "token_embedding.").replace(".mixer_norm.", ".attn_norm.")
        legacy[k.replace(".mixer.", ".attn.")] = v
    assert "token_embedding.weight" in legacy and any(".attn_norm." in k for k in legacy)
    ck = tmp_path / "last.pt"
    torch.save({"model_config": old_cfg, "model_state_dict": legacy, "training_args": {}}, ck)
    convert_legacy.main([str(ck), str(tmp_path / "out")])
    loaded = load_model(tmp_path / "out", device="cpu")
    ids = torch.randint(0, 256, (1, 20))
    with torch.no_grad():
        assert torch.allclose(loaded(ids).hidden, model.eval()(ids).hidden)
    with pytest.raises(ValueError):
        convert_legacy.convert_config({**old_cfg, "dropout": 0.1})
    del tiny_model_config


def test_sweep_train_summary_and_report(tmp_path):
    from myk_llm_b200.train import sweep_train

    sweep_dir = tmp_path / "sw"
    for name, bpb, speed in (("a-s0", 1.10, 1e5), ("a-s1", 1.20, 1.2e5), ("b-s0", 1.00, 9e4)):
        d = sweep_dir / name
        d.mkdir(parents=True)
        (d / "config.yaml").write_text("steps: 100\n")
        recs = [{"step": 0, "params/total": 1000}] + [{"step": s, "perf/tokens_per_s": speed} for s in range(1, 100)]
        recs.append({"step": 100, "val/en/loss": 2.0, "val/en/bpb": bpb})
        (d / "metrics.jsonl").write_text("\n".join(json.dumps(r) for r in recs))
        s = sweep_train.summarize(d)
        assert s["step"] == s["steps"] == 100 and s["params"] == {"total": 1000}
        assert s["tokens_per_s"] == pytest.approx(speed)
        (d / "results.json").write_text(json.dumps(s))
    table = sweep_train.report(sweep_dir).splitlines()
    assert table[2].startswith("| b | 1 | 1.0000") and table[3].startswith("| a | 2 | 1.1500")
    assert sweep_train.summarize(tmp_path / "missing") is None


def test_mtp_acceptance_summary():
    from myk_llm_b200.infer.eval_mtp_acceptance import repeat_fraction, summarize

    part = {"accepted": np.array([[1, 1, 0, 0], [1, 0, 0, 0]], dtype=np.float32),
            "p_accepted": np.full((2, 4), 0.5, dtype=np.float32),
            "bytes": np.full((2, 4), 3.0, dtype=np.float32), "first_bytes": np.full(4, 2.0, dtype=np.float32)}
    s = summarize([part])
    assert s["positions"] == 4
    assert [r["a_k"] for r in s["rows"]] == [1.0, 0.5, 0.25]
    assert s["rows"][2]["tokens_per_iter"] == pytest.approx(1.75)
    assert s["rows"][2]["bytes_per_iter"] == pytest.approx(2 + 3 * 0.75)
    assert repeat_fraction([1, 2, 3, 4, 1, 2, 3, 4]) == pytest.approx(1 / 5)


def test_small_helpers(tmp_path, capsys):
    from myk_llm_b200.utils import aggregate, training_cost

    (tmp_path / "src" / "sub").mkdir(parents=True)
    (tmp_path / "src" / "a.py").write_text("A\n")
    (tmp_path / "src" / "sub" / "b.md").write_text("B\n")
    (tmp_path / "src" / "c.bin").write_bytes(b"\xff\xfe")
    taken = aggregate.aggregate(str(tmp_path / "src"), [".py", ".md"], str(tmp_path / "out.txt"), seed=0)
    assert len(taken) == 2 and sorted((tmp_path / "out.txt").read_text().split()) == ["A", "B"]
    assert training_cost.training_hours(100, 180) == pytest.approx(100e9 / 180e3 / 3600)
    training_cost.main(["0.036", "10", "--gpus", "8", "--usd-per-gpu-hour", "2"])
    out = capsys.readouterr().out
    assert "1.00 hours" in out and "GPU-hours: 8.0" in out and "$16" in out
    assert sys.modules["myk_llm_b200.utils.aggregate"] is aggregate
