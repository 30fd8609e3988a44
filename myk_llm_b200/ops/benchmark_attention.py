"""Speed of this framework's FlashAttention (tcgen05) against the reference's Triton
FlashAttention (``baseline/_ref``, when installed), PyTorch SDPA (flash and cuDNN backends,
plain causal shapes) and FlexAttention (windows, packed documents): forward and forward +
backward, bf16, one GPU.  TFLOP/s count only visible (query, key) pairs; the backward
counts as 2.5x the forward (the reference's convention)::

    python -m myk_llm_b200.ops.benchmark_attention [--markdown]

Shapes: the reference's own benchmark list (``scripts/benchmark_attention.py:22-30``) and
this framework's training shapes (200M and 1B-hybrid layers).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.nn.functional as F

# (batch, seq, heads, kv_heads, head_dim, sliding window or None, document lengths or None)
REFERENCE_SHAPES = [
    (8, 2048, 8, 2, 128, None, None),
    (8, 2048, 8, 2, 128, 512, None),
    (8, 2048, 8, 2, 128, None, [300, 700, 48, 1000]),
    (2, 8192, 8, 2, 128, None, None),
    (16, 1024, 4, 4, 64, None, None),
    (16, 1024, 4, 4, 64, 256, None),
]
OUR_SHAPES = [
    (8, 4096, 16, 4, 64, None, None),       # 200M global layer, whole rows
    (8, 4096, 16, 4, 64, None, [1000, 300, 2048, 748]),  # 200M with packed documents
    (2, 8192, 16, 4, 128, None, None),      # 1B hybrid attention layer
]
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def visible_pairs(L: int, window: int | None, docs: list[int] | None) -> float:
    if docs:
        return sum(visible_pairs(d, window, None) for d in docs)
    return float(sum(min(i + 1, window or L) for i in range(L)))


def _bench(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _reference_ops():
    """The reference's attention entry points, or None when it is not installed."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "myk_llm")):
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        from myk_llm.ops import flash_attn_func, flash_attn_varlen_func
    except Exception:  # noqa: BLE001
        return None
    return flash_attn_func, flash_attn_varlen_func


def _arms(q, k, v, win, docs, B, L, ours, ref):
    """name -> (forward callable, inputs that get gradients)."""
    window = (win - 1, 0) if win else (-1, 0)
    arms = {}
    if docs:
        cu = torch.tensor([0] + list(torch.tensor(docs * B).cumsum(0)), dtype=torch.int32, device="cuda")
        flat = tuple(t.detach().reshape(B * L, t.shape[2], t.shape[3]).requires_grad_() for t in (q, k, v))
        arms["ours"] = (lambda: ours[1](*flat, cu, cu, max(docs), max(docs), causal=True, window_size=window), flat)
        if ref is not None:
            arms["reference triton"] = (lambda: ref[1](*flat, cu, cu, L, L, causal=True,
                                                       window_size=(win - 1, 0) if win else (-1, -1)), flat)
    else:
        arms["ours"] = (lambda: ours[0](q, k, v, causal=True, window_size=window), (q, k, v))
        if ref is not None:
            arms["reference triton"] = (lambda: ref[0](q, k, v, causal=True,
                                                       window_size=(win - 1, 0) if win else (-1, -1)), (q, k, v))
    qt, kt, vt = (t.detach().transpose(1, 2).requires_grad_() for t in (q, k, v))
    if win is None and docs is None:
        from torch.nn.attention import SDPBackend, sdpa_kernel

        for name, backend in (("sdpa flash", SDPBackend.FLASH_ATTENTION), ("sdpa cudnn", SDPBackend.CUDNN_ATTENTION)):
            def run(backend=backend):
                with sdpa_kernel(backend):
                    return F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True)
            arms[name] = (run, (qt, kt, vt))
    flex = _flex(qt, kt, vt, L, win, docs)
    if flex is not None:
        arms["flex"] = (flex, (qt, kt, vt))
    return arms


def _flex(qt, kt, vt, L, win, docs):
    try:
        from torch.nn.attention.flex_attention import create_block_mask, flex_attention
    except ImportError:
        return None
    doc = None
    if docs:
        doc = torch.repeat_interleave(torch.arange(len(docs), device=qt.device), torch.tensor(docs, device=qt.device))

    def mask(b, h, qi, ki):
        m = qi >= ki
        if win:
            m = m & (qi - ki < win)
        if doc is not None:
            m = m & (doc[qi] == doc[ki])
        return m

    block = create_block_mask(mask, None, None, L, L, device=qt.device)
    compiled = torch.compile(flex_attention, dynamic=False)
    return lambda: compiled(qt, kt, vt, block_mask=block, enable_gqa=True)


def measure(shape, reps: int, ours, ref) -> dict:
    B, L, H, KV, D, win, docs = shape
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(B, L, h, D, device="cuda", dtype=torch.bfloat16, generator=g).requires_grad_()
               for h in (H, KV, KV))
    flops = 4 * B * H * D * visible_pairs(L, win, docs)
    row = {"shape": list(shape)}
    for name, (fwd, inputs) in _arms(q, k, v, win, docs, B, L, ours, ref).items():
        try:
            out = fwd()
            do = torch.randn_like(out)
            t_fwd = _bench(fwd, reps)
            t_all = _bench(lambda: torch.autograd.grad(fwd(), inputs, do), reps)
            row[name] = {"fwd_ms": t_fwd, "fwd_tflops": flops / t_fwd / 1e9,
                         "fwdbwd_ms": t_all, "fwdbwd_tflops": 3.5 * flops / t_all / 1e9}
        except Exception as err:  # noqa: BLE001  (a backend this build lacks)
            row[name] = {"error": f"{type(err).__name__}: {str(err)[:100]}"}
    return row


def markdown(rows: list[dict]) -> str:
    out = []
    for row in rows:
        B, L, H, KV, D, win, docs = row["shape"]
        out.append(f"\n{B} x {L}, heads {H}/{KV} x {D}, window {win}, documents {docs}\n")
        out.append("| kernel | fwd ms | fwd TFLOP/s | fwd+bwd ms | fwd+bwd TFLOP/s |\n|---|---|---|---|---|")
        for name, r in row.items():
            if name == "shape":
                continue
            if "error" in r:
                out.append(f"| {name} | {r['error']} | | | |")
            else:
                out.append(f"| {name} | {r['fwd_ms']:.3f} | {r['fwd_tflops']:.0f} | {r['fwdbwd_ms']:.3f} | "
                           f"{r['fwdbwd_tflops']:.0f} |")
    return "\n".join(out)


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--markdown", action="store_true")
    args = ap.parse_args(argv)
    from . import flash_attn_func, flash_attn_varlen_func

    ours, ref = (flash_attn_func, flash_attn_varlen_func), _reference_ops()
    rows = []
    for shape in REFERENCE_SHAPES + OUR_SHAPES:
        rows.append(measure(shape, args.reps, ours, ref))
        if not args.markdown:
            print(json.dumps(rows[-1]), flush=True)
    if args.markdown:
        print(markdown(rows))


if __name__ == "__main__":
    main()
