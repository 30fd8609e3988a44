"""MXFP8: the block-scaling statement (CPU), model conversion rules, and on the GPU the
quantize kernel (bit-exact against the statement), the block-scaled tcgen05 GEMM
against fp32 math on the dequantized operands, and MXFP8 linears / a training step
tracking bf16."""

import pytest
import torch
import torch.nn as nn

from myk_llm_b200.ops import mxfp8


def test_block_exponents_are_exact_rceil():
    x = torch.zeros(2, 64)
    x[0, :32] = 448.0          # amax / max = 1 -> e = 0
    x[0, 32:] = 448.0 * 1.001  # just above -> e = 1
    x[1, :32] = 3.5            # 3.5 / 448 = 2^-7 -> e = -7
    e = mxfp8.block_exponents(x, "e4m3")
    assert e.tolist() == [[0, 1], [-7, -127]]
    q, e = mxfp8.quantize_ref(torch.randn(64, 256) * 50, "e4m3")
    assert q.float().abs().max() <= 448.0


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_quantization_error_is_bounded(fmt):
    x = torch.randn(32, 128) * torch.logspace(-3, 3, 32)[:, None]
    q, e = mxfp8.quantize_ref(x, fmt)
    err = (mxfp8.dequantize_ref(q, e) - x).abs()
    bound = (2.0 ** -3 if fmt == "e4m3" else 2.0 ** -2) * x.reshape(32, 4, 32).abs().amax(-1).repeat_interleave(32, -1)
    assert torch.all(err <= bound)


def test_conversion_keeps_parameters_and_rules():
    from conftest import tiny_model_config
    from myk_llm_b200.models import MykLLM
    from myk_llm_b200.parallel.distributed import convert_float8

    model = MykLLM(tiny_model_config(layer_pattern="GD", ffn={"multiplier": 2.0, "multiple_of": 64}))
    before = {k: v.clone() for k, v in model.state_dict().items()}
    n = convert_float8(model, "mxfp8", skip_down_proj=True, grad_dtype="e5m2")
    assert n > 0
    assert model.state_dict().keys() == before.keys()
    for name, mod in model.named_modules():
        if name == "lm_head" or name.endswith((".a_proj", ".b_proj", ".down_proj")):
            assert not isinstance(mod, mxfp8.MXFP8Linear), name
        if isinstance(mod, mxfp8.MXFP8Linear):
            assert mod.weight._mykb_mxfp8 == "e5m2"
    with pytest.raises(ValueError):
        convert_float8(nn.Sequential(nn.Linear(64, 64)), "blockwise")


# ------------------------------------------------------------------------------ GPU
def _mk(r, c, seed=0, outlier=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(r, c, device="cuda", generator=g) * torch.logspace(-2, 2, c, device="cuda")[None, :]
    if outlier:
        x[r // 3, c // 5] = 2e5
    return x.bfloat16()


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("shape", [(128, 128), (256, 384), (100, 256)])
def test_quantize_kernel_is_bit_exact(fmt, shape):
    r, c = shape
    x = _mk(r, c)
    dim1 = r % 128 == 0
    out = mxfp8.mx_quantize(x, fmt, dim0=True, dim1=dim1)
    q_ref, e_ref = mxfp8.quantize_ref(x, fmt)
    q0, s0 = out[0], out[1]
    assert torch.equal(q0, q_ref.view(torch.uint8))
    assert torch.equal(mxfp8.atoms_to_exponents(s0, r, c), e_ref.long())
    if dim1:
        qt_ref, et_ref = mxfp8.quantize_ref(x.t().contiguous(), fmt)
        assert torch.equal(out[2], qt_ref.view(torch.uint8))
        assert torch.equal(mxfp8.atoms_to_exponents(out[3], c, r), et_ref.long())


def _dequant(q_u8, atoms, rows, k, fmt):
    e = mxfp8.atoms_to_exponents(atoms, rows, k)
    return mxfp8.dequantize_ref(q_u8.view(mxfp8.TORCH_FP8[fmt]), e)


@pytest.mark.gpu
@pytest.mark.parametrize("mnk", [(128, 128, 128), (256, 384, 512), (200, 136, 256), (1024, 1536, 1024)])
@pytest.mark.parametrize("fmts", [("e4m3", "e4m3"), ("e5m2", "e4m3"), ("e5m2", "e5m2")])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_block_scaled_gemm_matches_dequantized_math(mnk, fmts, out_dtype):
    m, n, k = mnk
    a, b = _mk(m, k, 1), _mk(n, k, 2)
    qa, sa = mxfp8.mx_quantize(a, fmts[0])
    qb, sb = mxfp8.mx_quantize(b, fmts[1])
    ref = _dequant(qa, sa, m, k, fmts[0]) @ _dequant(qb, sb, n, k, fmts[1]).t()
    out = mxfp8.mx_gemm(qa, sa, fmts[0], qb, sb, fmts[1], out_dtype=out_dtype)
    torch.cuda.synchronize()
    err = (out.float() - ref).abs().max() / ref.abs().max()
    assert err < (1e-2 if out_dtype == torch.bfloat16 else 1e-4), float(err)
    acc = torch.ones(m, n, device="cuda")
    mxfp8.mx_gemm(qa, sa, fmts[0], qb, sb, fmts[1], out=acc, accumulate=True)
    assert ((acc - 1 - ref).abs().max() / ref.abs().max()) < 1e-4


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).item()


@pytest.mark.gpu
@pytest.mark.parametrize("grad_fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("rows,outlier", [(512, False), (300, True)])
def test_mx_linear_tracks_bf16(grad_fmt, rows, outlier):
    from myk_llm_b200.ops.linear import linear

    x = _mk(rows, 256, 3, outlier=outlier).requires_grad_(True)
    w = (torch.randn(384, 256, device="cuda") * 0.05).requires_grad_(True)
    y = mxfp8.mx_linear(x, w, grad_fmt)
    dy = torch.randn_like(y)
    y.backward(dy)
    x2 = x.detach().clone().requires_grad_(True)
    w2 = w.detach().clone().requires_grad_(True)
    y2 = linear(x2, w2)
    y2.backward(dy)
    assert _cos(y, y2) > 0.998
    assert _cos(x.grad, x2.grad) > 0.99
    assert _cos(w.grad, w2.grad) > 0.99


@pytest.mark.gpu
def test_training_step_with_converted_model_tracks_bf16():
    from conftest import tiny_model_config
    from myk_llm_b200.models import MykLLM
    from myk_llm_b200.parallel.distributed import convert_float8

    torch.manual_seed(0)
    cfg = tiny_model_config(hidden_size=256, layer_pattern="G", ffn={"multiplier": 2.0, "multiple_of": 128},
                            attention={"num_heads": 4, "num_kv_heads": 2, "head_dim": 64})
    base = MykLLM(cfg).cuda()
    mx = MykLLM(cfg).cuda()
    mx.load_state_dict(base.state_dict())
    assert convert_float8(mx, "mxfp8") > 0
    ids = torch.randint(0, cfg.vocab_size, (4, 128), device="cuda")
    losses = []
    for model in (base, mx):
        hid = model(ids).hidden
        loss = torch.nn.functional.cross_entropy(model.logits(hid).float().flatten(0, 1)[:-1], ids.flatten()[1:])
        loss.backward()
        losses.append(loss.item())
    assert abs(losses[0] - losses[1]) / losses[0] < 0.01
    for (n1, p1), (n2, p2) in zip(base.named_parameters(), mx.named_parameters()):
        if p1.grad is not None and p1.grad.abs().sum() > 0:
            assert _cos(p1.grad, p2.grad) > 0.98, n1
