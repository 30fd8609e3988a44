"""Streaming loader: packing, seam masking, token-balanced interleave and exact resume,
over local jsonl files with a character tokenizer (no network)."""

import json
from types import SimpleNamespace

import numpy as np
import pytest

pytest.importorskip("datasets")

from myk_llm_b200.data.config import IGNORE_INDEX, DataConfig, SourceConfig  # noqa: E402
from myk_llm_b200.data.filters import DocFilter  # noqa: E402
from myk_llm_b200.data.streaming import PackedStreamDataset, StreamLoader, take_windows  # noqa: E402

EOS = 0


class CharTokenizer:
    def encode_batch(self, texts, add_special_tokens=False):
        return [SimpleNamespace(ids=[1 + (ord(c) % 200) for c in t]) for t in texts]


def _corpus(tmp_path, name, n, prefix):
    p = tmp_path / f"{name}.jsonl"
    rng = np.random.default_rng(len(name))
    with open(p, "w") as f:
        for i in range(n):
            length = int(rng.integers(5, 60))
            f.write(json.dumps({"text": f"{prefix}{i} " + "x" * length}) + "\n")
    return str(p)


def _config(tmp_path, weights=(1.0,), seq_len=64):
    sources = [SourceConfig(name=f"s{k}", weight=w, path=_corpus(tmp_path, f"s{k}", 200, chr(97 + k)), curated=True)
               for k, w in enumerate(weights)]
    return DataConfig(kind="stream", seq_len=seq_len, micro_batch_size=2, sources=sources, shuffle_buffer=16,
                      num_workers=0, doc_filter=DocFilter())


def test_windows_are_packed_with_seams_masked(tmp_path):
    cfg = _config(tmp_path)
    rows = take_windows(cfg, EOS, 6, seed=0, tokenizer=CharTokenizer())
    for r in rows:
        assert r["input_ids"].shape == (64,) and r["targets"].shape == (64,)
        assert int(r["seqlens"].sum()) == 64
        # targets equal the next input except across a document seam
        same = r["targets"][:-1] == r["input_ids"][1:]
        masked = r["targets"][:-1] == IGNORE_INDEX
        assert np.all(same | masked)
        # every masked target is at the end of a document segment
        ends = np.cumsum(r["seqlens"]) - 1
        assert set(np.flatnonzero(r["targets"] == IGNORE_INDEX)) <= set(ends.tolist())


def test_token_balanced_interleave(tmp_path):
    cfg = _config(tmp_path, weights=(3.0, 1.0))
    ds = PackedStreamDataset(cfg, EOS, tokenizer=CharTokenizer())
    it = iter(ds)
    for _ in range(40):
        next(it)
    share = ds.packer.consumed / ds.packer.consumed.sum()
    assert abs(share[0] - 0.75) < 0.05


def test_state_dict_resumes_exactly(tmp_path):
    cfg = _config(tmp_path, weights=(1.0, 2.0))
    a = PackedStreamDataset(cfg, EOS, tokenizer=CharTokenizer())
    it = iter(a)
    for _ in range(7):
        next(it)
    state = a.state_dict()
    expect = [next(it) for _ in range(5)]
    b = PackedStreamDataset(cfg, EOS, tokenizer=CharTokenizer())
    b.load_state_dict(state)
    got = [w for _, w in zip(range(5), iter(b))]
    for x, y in zip(expect, got):
        assert np.array_equal(x["input_ids"], y["input_ids"]) and np.array_equal(x["seqlens"], y["seqlens"])


def test_stream_loader_batches(tmp_path):
    cfg = _config(tmp_path)
    loader = StreamLoader(cfg, EOS, tokenizer=CharTokenizer())
    b = loader.next_batch()
    assert tuple(b.input_ids.shape) == (2, 64) and len(b.seqlens) == 2
    state = loader.state_dict()
    assert state["kind"] == "stream"
