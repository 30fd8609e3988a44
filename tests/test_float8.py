"""Per-tensor / per-row float8 linears: the scaling statements on the CPU, model conversion
rules, and on the GPU the cuBLASLt float8 GEMMs against fp32 math on the same quantised
operands plus a training step of a converted model."""

import pytest
import torch
import torch.nn as nn

from myk_llm_b200.ops import float8 as f8


def _ref_linear(x, w, recipe):
    """fp32 statement of the three GEMMs on the quantised operands."""
    rowwise = recipe != "tensorwise"

    def dq(t, dtype, rw):
        q, s = f8.quantize(t, dtype, rw)
        return q.float() * s

    y = dq(x, f8.E4M3, rowwise) @ dq(w, f8.E4M3, rowwise).t()
    return y


def test_quantize_tensorwise_and_rowwise():
    torch.manual_seed(0)
    x = torch.randn(64, 128) * torch.logspace(-2, 2, 64)[:, None]
    q, s = f8.quantize(x, f8.E4M3, False)
    assert q.dtype == f8.E4M3 and s.numel() == 1
    assert torch.isclose(s, x.abs().max() / 448.0)
    assert (q.float().abs().max() - 448.0).abs() < 1e-3
    q, s = f8.quantize(x, f8.E4M3, True)
    assert s.shape == (64, 1)
    # power-of-two scales that keep every row inside the E4M3 range
    assert torch.equal(torch.log2(s), torch.round(torch.log2(s)))
    assert (q.float().abs().amax(dim=1) <= 448.0).all()
    assert (x.abs().amax(dim=1, keepdim=True) / s > 224.0 - 1e-3).all()
    rel = ((q.float() * s - x).abs() / x.abs().amax(dim=1, keepdim=True)).max()
    assert rel < 2 ** -4


@pytest.mark.parametrize("recipe", f8.RECIPES)
def test_fp8_linear_cpu_statement(recipe):
    torch.manual_seed(1)
    x = torch.randn(4, 16, 64, requires_grad=True)
    w = nn.Parameter(torch.randn(32, 64) * 0.1)
    y = f8.fp8_linear(x, w, recipe)
    assert y.shape == (4, 16, 32) and y.dtype == torch.bfloat16
    ref = _ref_linear(x.detach().reshape(-1, 64), w.detach(), recipe)
    torch.testing.assert_close(y.float().reshape(-1, 32), ref, atol=2e-2, rtol=1e-2)
    dy = torch.randn(4, 16, 32)
    y.backward(dy.to(y.dtype))
    # gradients agree with fp32 math to float8 accuracy
    xf, wf = x.detach().reshape(-1, 64), w.detach()
    g = dy.reshape(-1, 32)
    dx_ref, dw_ref = g @ wf, g.t() @ xf
    rel_dx = (x.grad.reshape(-1, 64).float() - dx_ref).norm() / dx_ref.norm()
    rel_dw = (w.grad.float() - dw_ref).norm() / dw_ref.norm()
    assert rel_dx < 0.1 and rel_dw < 0.1
    if recipe == "rowwise_with_gw_hp":
        assert rel_dw < 0.01   # bf16 weight gradient


def test_fp8_main_grad_accumulates():
    torch.manual_seed(2)
    x = torch.randn(32, 64)
    w = nn.Parameter(torch.randn(32, 64) * 0.1)
    w.main_grad = torch.zeros(32, 64)
    for _ in range(2):
        f8.fp8_linear(x, w, "rowwise").sum().backward()
    assert w.grad is None and w.main_grad.abs().sum() > 0
    w2 = nn.Parameter(w.detach().clone())
    f8.fp8_linear(x, w2, "rowwise").sum().backward()
    torch.testing.assert_close(w.main_grad, 2 * w2.grad.float())


def test_convert_float8_rules():
    from tests.conftest import tiny_model_config
    from myk_llm_b200.models import MykLLM
    from myk_llm_b200.parallel.distributed import convert_float8

    model = MykLLM(tiny_model_config(layer_pattern="GD", tie_embeddings=False))
    n = convert_float8(model, "tensorwise", skip_down_proj=True)
    assert n > 0
    for name, mod in model.named_modules():
        if name == "lm_head" or name.endswith((".a_proj", ".b_proj", ".down_proj")):
            assert not isinstance(mod, f8.Float8Linear), name
        if isinstance(mod, f8.Float8Linear):
            assert mod.weight._mykb_fp8 == "tensorwise"
    with pytest.raises(ValueError):
        convert_float8(model, "blockwise")


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(256, 512), (4096, 1024), (80, 200), (1040, 3072)])
@pytest.mark.parametrize("dtype", [f8.E4M3, f8.E5M2])
def test_quantizer_kernels_match_statement(shape, dtype):
    """The fused quantisers reproduce the PyTorch statement bit for bit."""
    from myk_llm_b200.ops._ext import ext

    torch.manual_seed(5)
    r, c = shape
    x = (torch.randn(r, c, device="cuda") * torch.logspace(-3, 3, r, device="cuda")[:, None]).to(torch.bfloat16)
    x[0, :8] = 0   # a partly zero row
    e5 = dtype == f8.E5M2
    for rowwise in (False, True):
        q, s = ext().fp8_quant_rows(x, e5, True) if rowwise else ext().fp8_quant_tensor(x, e5)
        qr, sr = f8.quantize(x, dtype, rowwise)
        assert q.dtype == dtype and s.shape == sr.shape
        assert torch.equal(s, sr)
        assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8))
    if r % 16 == 0:
        qt, st = ext().fp8_quant_cols_t(x, e5, True)
        qr, sr = f8.quantize(x.t().contiguous(), dtype, True)
        assert torch.equal(st, sr)
        assert torch.equal(qt.view(torch.uint8), qr.view(torch.uint8))


@pytest.mark.gpu
@pytest.mark.parametrize("recipe", f8.RECIPES)
def test_fp8_linear_gpu_matches_statement(recipe):
    torch.manual_seed(3)
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = nn.Parameter(torch.randn(384, 512, device="cuda") * 0.05)
    y = f8.fp8_linear(x, w, recipe)
    ref = _ref_linear(x.detach().float(), w.detach(), recipe)
    torch.testing.assert_close(y.float(), ref, atol=5e-2, rtol=2e-2)
    dy = torch.randn(256, 384, device="cuda", dtype=torch.bfloat16)
    y.backward(dy)
    xf, wf, g = x.detach().float(), w.detach(), dy.float()
    dx_ref, dw_ref = g @ wf, g.t() @ xf
    assert (x.grad.float() - dx_ref).norm() / dx_ref.norm() < 0.1
    assert (w.grad.float() - dw_ref).norm() / dw_ref.norm() < (0.01 if recipe == "rowwise_with_gw_hp" else 0.1)
    # the CPU statement of the same recipe agrees with the GPU one to accumulation order
    xc = x.detach().cpu().requires_grad_(True)
    wc = nn.Parameter(w.detach().cpu())
    yc = f8.fp8_linear(xc, wc, recipe)
    torch.testing.assert_close(y.float().cpu(), yc.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("recipe", f8.RECIPES)
def test_fp8_model_step_tracks_bf16(recipe):
    from tests.conftest import tiny_model_config
    from myk_llm_b200.models import MykLLM
    from myk_llm_b200.parallel.distributed import convert_float8

    torch.manual_seed(4)
    cfg = tiny_model_config(hidden_size=256, layer_pattern="G", ffn={"multiplier": 2.0, "multiple_of": 128},
                            attention={"num_heads": 4, "num_kv_heads": 2, "head_dim": 64})
    base = MykLLM(cfg).cuda()
    fp8 = MykLLM(cfg).cuda()
    fp8.load_state_dict(base.state_dict())
    assert convert_float8(fp8, recipe) > 0
    ids = torch.randint(0, cfg.vocab_size, (4, 128), device="cuda")
    losses = []
    for model in (base, fp8):
        hid = model(ids).hidden
        loss = torch.nn.functional.cross_entropy(model.logits(hid).float().flatten(0, 1)[:-1], ids.flatten()[1:])
        loss.backward()
        losses.append(loss.item())
    assert abs(losses[0] - losses[1]) / losses[0] < 0.01
    for (n1, p1), (_, p2) in zip(base.named_parameters(), fp8.named_parameters()):
        if p1.grad is not None and p1.grad.abs().sum() > 0:
            cos = torch.nn.functional.cosine_similarity(p1.grad.flatten().float(), p2.grad.flatten().float(), dim=0)
            assert cos > 0.97, n1
