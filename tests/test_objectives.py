"""Training objectives on CPU against plain PyTorch statements: MTP target windows, and the
distillation KL whose gradients are produced during forward (value and both gradients
against autograd through a direct log-softmax statement)."""

import torch
import torch.nn.functional as F

from myk_llm_b200.data.config import IGNORE_INDEX
from myk_llm_b200.train.objectives import distillation_kl_sum, mtp_targets


def _mtp_statement(targets, depth):
    out = torch.full_like(targets, IGNORE_INDEX)
    b, s = targets.shape
    for i in range(b):
        for j in range(s):
            span = targets[i, j:j + depth + 1]
            if span.numel() == depth + 1 and bool((span != IGNORE_INDEX).all()):
                out[i, j] = targets[i, j + depth]
    return out


def test_mtp_targets_match_the_window_rule():
    g = torch.Generator().manual_seed(0)
    t = torch.randint(0, 50, (3, 40), generator=g)
    t[torch.rand(3, 40, generator=g) < 0.2] = IGNORE_INDEX
    for depth in (1, 2, 3):
        assert torch.equal(mtp_targets(t, depth), _mtp_statement(t, depth))


def test_distillation_kl_value_and_gradients():
    g = torch.Generator().manual_seed(1)
    h = torch.randn(37, 16, generator=g, requires_grad=True)
    w = torch.randn(30, 16, generator=g, requires_grad=True)
    th, tw = torch.randn(37, 12, generator=g), torch.randn(30, 12, generator=g)
    valid = torch.rand(37, generator=g) > 0.3
    temp = 2.0
    student = F.log_softmax(h @ w.t() / temp, -1)
    teacher = F.log_softmax(th @ tw.t() / temp, -1)
    ref = ((teacher.exp() * (teacher - student)).sum(-1) * valid.float()).sum() * temp ** 2
    ref.backward()
    gh, gw = h.grad.clone(), w.grad.clone()
    h.grad = w.grad = None
    got = distillation_kl_sum(h, w, th, tw, valid, temp, 8)
    (0.5 * got).backward()
    assert torch.allclose(got, ref, rtol=1e-5)
    assert torch.allclose(h.grad, 0.5 * gh, atol=1e-5)
    assert torch.allclose(w.grad, 0.5 * gw, atol=1e-5)
