"""Lazy (sparse-Adam) n-gram tables: LazyAdam semantics, closed-form catch-up against
dense AdamW, checkpoint round trip and export, and the CUDA kernels against the torch
statement of the same update."""

import math

import pytest
import torch

from myk_llm_b200.models.config import NgramEmbeddingConfig
from myk_llm_b200.models.embeddings import NgramEmbedding
from myk_llm_b200.train.config import NgramOptimConfig
from myk_llm_b200.train.ngram_tables import SparseNgramTables

VOCAB = 50


def _module(seed=0, buckets=64, dim=8):
    torch.manual_seed(seed)
    m = NgramEmbedding(NgramEmbeddingConfig(orders=[2, 3], num_buckets=buckets, dim=dim), VOCAB, dim)
    for t in m.tables:
        torch.nn.init.normal_(t.weight, std=0.1)
    return m


def _batches(steps, seed=1, length=12):
    g = torch.Generator().manual_seed(seed)
    # a small token range so that rows repeat across steps, with gaps
    return [torch.randint(0, 6 + 3 * (s % 3), (2, length), generator=g) for s in range(steps)]


def _tables(module, device="cpu", **cfg):
    c = NgramOptimConfig(update="lazy", **cfg)
    return SparseNgramTables(module, c, lr=1e-2, betas=(0.9, 0.95), eps=1e-8, device=torch.device(device),
                             max_rows_per_step=10_000)


def _train(tables, module, batches, target_seed=3):
    g = torch.Generator().manual_seed(target_seed)
    for x in batches:
        tables.begin_step([x])
        out = module.lookup(x, None)
        target = torch.randn(out.shape, generator=g).to(out.device)
        ((out - target) ** 2).sum().backward()
        tables.step()


def test_lazy_adam_updates_only_touched_rows():
    mod = _module()
    before = torch.cat([t.weight.detach().clone() for t in mod.tables])
    tabs = _tables(mod)
    x = torch.tensor([[1, 2, 3, 1, 2, 3]])
    touched = torch.unique(mod.row_ids(x).flatten())
    _train(tabs, mod, [x])
    after = tabs.weight
    mask = torch.zeros(after.size(0), dtype=torch.bool)
    mask[touched] = True
    assert not torch.equal(after[mask], before[mask])
    assert torch.equal(after[~mask], before[~mask])
    assert torch.all(tabs.state[3][touched] == 1) and torch.all(tabs.state[3][~mask] == 0)


def _dense_adamw(module, batches, wd, start, rowwise=False, target_seed=3):
    """Dense AdamW (every row, every step, zero gradients on untouched rows) from global
    step ``start``."""
    b1, b2, lr, eps = 0.9, 0.95, 1e-2, 1e-8
    weight = torch.cat([t.weight.detach().clone() for t in module.tables])
    m = torch.zeros_like(weight)
    v = torch.zeros(weight.size(0), 1) if rowwise else torch.zeros_like(weight)
    g = torch.Generator().manual_seed(target_seed)
    for i, x in enumerate(batches, start=1):
        t = start + i
        leaf = weight.clone().requires_grad_()
        out = torch.nn.functional.embedding(module.row_ids(x), leaf).sum(0)
        target = torch.randn(out.shape, generator=g)
        ((out - target) ** 2).sum().backward()
        grad = leaf.grad
        weight = weight * (1 - lr * wd)
        m = m + (1 - b1) * (grad - m)
        v = v * b2 + (1 - b2) * (grad.square().mean(1, keepdim=True) if rowwise else grad * grad)
        weight = weight - lr / (1 - b1 ** t) * m / (v.sqrt() / math.sqrt(1 - b2 ** t) + eps)
    return weight


@pytest.mark.parametrize("wd", [0.0, 0.1])
@pytest.mark.parametrize("rowwise", [False, True])
def test_catch_up_matches_dense_adamw(wd, rowwise):
    """Late in training (bias corrections ~1) lazy Adam with catch_up equals dense AdamW up
    to eps; without catch_up the skipped rows fall behind."""
    start = 10_000
    batches = _batches(10)
    dense = _dense_adamw(_module(), batches, wd, start, rowwise)
    kw = dict(weight_decay=wd, second_moment="rowwise" if rowwise else "elementwise")
    mod = _module()
    tabs = _tables(mod, catch_up=True, **kw)
    tabs.step_count = start
    tabs.state[3].fill_(start)
    _train(tabs, mod, batches)
    got = tabs.export_weights()
    got = torch.cat([got[f"embed.ngram.tables.{k}.weight"] for k in range(2)])
    torch.testing.assert_close(got, dense, rtol=1e-4, atol=1e-6)
    plain_mod = _module()
    plain = _tables(plain_mod, catch_up=False, **kw)
    plain.step_count = start
    _train(plain, plain_mod, batches)
    assert (plain.weight - dense).abs().max() > 100 * (got - dense).abs().max()
    with torch.no_grad():  # no-grad lookups see the caught-up rows
        x = batches[0]
        torch.testing.assert_close(mod.lookup(x, None),
                                   torch.nn.functional.embedding(mod.row_ids(x), dense).sum(0), rtol=1e-4, atol=1e-6)


def test_rowwise_second_moment_runs_and_differs():
    batches = _batches(4)
    a, b = _module(), _module()
    ta, tb = _tables(a), _tables(b, second_moment="rowwise")
    _train(ta, a, batches)
    _train(tb, b, batches)
    assert tb.exp_avg_sq.dim() == 1
    assert not torch.allclose(ta.weight, tb.weight)


def test_no_grad_lookup_reads_current_tables():
    mod = _module()
    tabs = _tables(mod)
    x = torch.tensor([[4, 5, 6]])
    _train(tabs, mod, [x])
    with torch.no_grad():
        out = mod.lookup(x, None)
    ids = mod.row_ids(x)
    ref = torch.nn.functional.embedding(ids, tabs.weight).sum(0)
    torch.testing.assert_close(out, ref)


def test_state_dict_round_trip_and_export(tmp_path):
    mod = _module()
    tabs = _tables(mod, catch_up=True)
    _train(tabs, mod, _batches(3))
    tabs.save(tmp_path)
    mod2 = _module(seed=9)
    tabs2 = _tables(mod2, catch_up=True)
    tabs2.load(tmp_path)
    for a, b in zip(tabs.state, tabs2.state):
        assert torch.equal(a, b)
    assert tabs2.step_count == tabs.step_count == 3
    ex = tabs.export_weights()
    assert set(ex) == {"embed.ngram.tables.0.weight", "embed.ngram.tables.1.weight"}
    assert ex["embed.ngram.tables.0.weight"].shape == (64, 8)


def test_begin_step_twice_is_an_error():
    mod = _module()
    tabs = _tables(mod)
    tabs.begin_step([torch.tensor([[1, 2]])])
    with pytest.raises(RuntimeError):
        tabs.begin_step([torch.tensor([[1, 2]])])


@pytest.mark.gpu
@pytest.mark.parametrize("placement", ["gpu", "host"])
@pytest.mark.parametrize("rowwise", [False, True])
def test_cuda_kernels_match_torch_statement(placement, rowwise):
    batches = _batches(8)
    cpu_mod = _module()
    cpu = _tables(cpu_mod, catch_up=True, weight_decay=0.05,
                  second_moment="rowwise" if rowwise else "elementwise")
    _train(cpu, cpu_mod, batches)
    gpu_mod = _module().cuda()
    gpu = _tables(gpu_mod, device="cuda", placement=placement, catch_up=True, weight_decay=0.05,
                  second_moment="rowwise" if rowwise else "elementwise")
    assert gpu.weight.is_cuda == (placement == "gpu")
    _train(gpu, gpu_mod, [b.cuda() for b in batches])
    torch.cuda.synchronize()
    for a, b in zip(cpu.state, gpu.state):
        torch.testing.assert_close(b.cpu(), a, rtol=1e-5, atol=1e-6)
