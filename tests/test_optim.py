"""Optimizers on CPU: Muon matches the per-matrix reference statement, AdamW matches
torch.optim.AdamW, schedules, parameter grouping."""

import math

import pytest
import torch

from myk_llm_b200.train.config import ScheduleConfig
from myk_llm_b200.train.optim import AdamW, Muon, lr_multiplier, lr_ratio, newton_schulz_orthogonalize, split_parameters


def test_adamw_matches_torch():
    torch.manual_seed(0)
    p1 = torch.nn.Parameter(torch.randn(10, 7))
    p2 = torch.nn.Parameter(p1.detach().clone())
    o1 = AdamW([p1], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    o2 = torch.optim.AdamW([p2], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for _ in range(5):
        g = torch.randn(10, 7)
        p1.grad, p2.grad = g.clone(), g.clone()
        o1.step()
        o2.step()
    assert torch.allclose(p1, p2, atol=1e-6)
    assert set(o1.state[p1]) == {"step", "exp_avg", "exp_avg_sq"}


def test_muon_matches_reference_statement():
    torch.manual_seed(1)
    p = torch.nn.Parameter(torch.randn(16, 32))
    ref = p.detach().clone()
    buf = torch.zeros_like(ref)
    opt = Muon([p], lr=0.02, weight_decay=0.1, momentum=0.95, nesterov=True, ns_steps=5)
    for _ in range(3):
        g = torch.randn(16, 32)
        p.grad = g.clone()
        opt.step()
        buf.lerp_(g, 0.05)
        u = g.lerp(buf, 0.95)
        o = newton_schulz_orthogonalize(u, 5)
        ref.mul_(1 - 0.02 * 0.1)
        ref.add_(o.float(), alpha=-0.02 * lr_ratio(ref.shape, "match_rms_adamw"))
    assert torch.allclose(p, ref, atol=1e-5)
    assert "momentum_buffer" in opt.state[p]


def test_schedules():
    c = ScheduleConfig(kind="wsd", warmup_ratio=0.1, decay_ratio=0.2, min_lr_ratio=0.1)
    assert lr_multiplier(5, 100, c) == 0.5
    assert lr_multiplier(50, 100, c) == 1.0
    assert abs(lr_multiplier(100, 100, c) - 0.1) < 1e-9
    cos = ScheduleConfig(kind="cosine", warmup_ratio=0.0, min_lr_ratio=0.0)
    assert abs(lr_multiplier(50, 100, cos) - 0.5 * (1 + math.cos(math.pi * 0.5))) < 1e-9


def test_split_parameters():
    from tests.conftest import tiny_model_config
    from myk_llm_b200.models import MykLLM

    m = MykLLM(tiny_model_config(layer_pattern="GD", tie_embeddings=False))
    g = split_parameters(m, use_muon=True)
    names = {id(p): n for n, p in m.named_parameters()}
    assert all(names[id(p)].startswith("layers") for p in g.muon)
    assert any(names[id(p)] == "lm_head.weight" for p in g.no_decay)
    assert any("conv1d" in names[id(p)] for p in g.decay)


@pytest.mark.parametrize("kind", ["adamw", "muon"])
def test_grad_scale_equals_prescaled_gradients(kind):
    """The clipping coefficient handed to the optimizer equals multiplying the gradients first."""
    torch.manual_seed(2)
    p1 = torch.nn.Parameter(torch.randn(16, 32))
    p2 = torch.nn.Parameter(p1.detach().clone())
    make = (lambda p: AdamW([p], lr=1e-2, weight_decay=0.1)) if kind == "adamw" else \
        (lambda p: Muon([p], lr=0.02, weight_decay=0.1))
    o1, o2 = make(p1), make(p2)
    for i in range(3):
        g = torch.randn(16, 32)
        scale = torch.tensor(0.3 + 0.2 * i)
        p1.grad, p2.grad = g.clone(), g * scale
        o1.grad_scale = scale
        o1.step()
        o1.grad_scale = None
        o2.step()
    assert torch.allclose(p1, p2, atol=1e-6)
