"""Speed of this framework's FlashAttention (tcgen05) against PyTorch SDPA (plain causal
shapes) and FlexAttention (windows, packed documents), forward and forward + backward,
on the shapes the configs train with (bf16, one GPU).  TFLOP/s count only visible
(query, key) pairs; the backward counts as 2.5x the forward::

    python -m myk_llm_b200.ops.benchmark_attention
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F

# (batch, seq, heads, kv_heads, head_dim, sliding window or None, document lengths or None)
SHAPES = [
    (8, 4096, 16, 4, 64, None, None),       # 200M global layer
    (8, 4096, 16, 4, 64, 1024, None),       # sliding-window layer
    (8, 4096, 16, 4, 64, None, [1000, 300, 2048, 748]),  # packed documents
    (2, 8192, 16, 4, 128, None, None),      # 1B hybrid attention layer
    (16, 1024, 4, 4, 64, None, None),       # lc testbed
]


def visible_pairs(L: int, window: int | None, docs: list[int] | None) -> float:
    if docs:
        return sum(visible_pairs(d, window, None) for d in docs)
    if window is None:
        return L * (L + 1) / 2
    w = window
    return sum(min(i + 1, w) for i in range(L))


def _flex(q, k, v, L, win, docs, B):
    """FlexAttention (compiled) over the same mask, or None where it is unavailable."""
    try:
        from torch.nn.attention.flex_attention import create_block_mask, flex_attention
    except ImportError:
        return None
    doc = None
    if docs:
        doc = torch.repeat_interleave(torch.arange(len(docs), device=q.device),
                                      torch.tensor(docs, device=q.device))

    def mask(b, h, qi, ki):
        m = qi >= ki
        if win:
            m = m & (qi - ki < win)
        if doc is not None:
            m = m & (doc[qi] == doc[ki])
        return m

    bm = create_block_mask(mask, None, None, L, L, device=q.device)
    fa = torch.compile(flex_attention)
    qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
    return lambda: fa(qt, kt, vt, block_mask=bm, enable_gqa=True)


def _bench(fn, reps: int = 10) -> float:
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


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args(argv)
    from . import flash_attn_func, flash_attn_varlen_func

    for B, L, H, KV, D, win, docs in SHAPES:
        q = torch.randn(B, L, H, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn(B, L, KV, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        v = torch.randn(B, L, KV, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        flops = 4 * B * H * D * visible_pairs(L, win, docs)
        row = {"shape": [B, L, H, KV, D, win, docs]}
        if docs:
            cu = torch.tensor([0] + list(torch.tensor(docs * B).cumsum(0)), dtype=torch.int32, device="cuda")
            qf, kf, vf = q.reshape(B * L, H, D), k.reshape(B * L, KV, D), v.reshape(B * L, KV, D)
            ours = lambda: flash_attn_varlen_func(qf, kf, vf, cu, cu, max(docs), max(docs), causal=True)  # noqa: E731
        else:
            ours = lambda: flash_attn_func(q, k, v, causal=True, window_size=(win - 1 if win else -1, 0))  # noqa: E731
        out = ours()
        do = torch.randn_like(out)
        row["ours_fwd_tflops"] = flops / _bench(ours, args.reps) / 1e9
        row["ours_fwdbwd_tflops"] = 3.5 * flops / _bench(
            lambda: torch.autograd.grad(ours(), (q, k, v), do), args.reps) / 1e9
        if win is None and docs is None:
            qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
            sdpa = lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True)  # noqa: E731
            try:
                row["sdpa_fwd_tflops"] = flops / _bench(sdpa, args.reps) / 1e9
                row["sdpa_fwdbwd_tflops"] = 3.5 * flops / _bench(
                    lambda: torch.autograd.grad(sdpa(), (q, k, v), do.transpose(1, 2)), args.reps) / 1e9
            except RuntimeError as err:  # a backend without GQA support on this build
                row["sdpa_error"] = str(err)[:80]
        flex = _flex(q, k, v, L, win, docs, B)
        if flex is not None:
            row["flex_fwd_tflops"] = flops / _bench(flex, args.reps) / 1e9
            row["flex_fwdbwd_tflops"] = 3.5 * flops / _bench(
                lambda: torch.autograd.grad(flex(), (q, k, v), do.transpose(1, 2)), args.reps) / 1e9
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
