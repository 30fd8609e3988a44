"""Per-kernel microbenchmarks: one small, fixed case per hot kernel, timed with CUDA
events (warm-up, then the mean of ``reps`` launches) and reported against the measured
roofline of the machine (``MEASURED_PEAKS.json`` at the repository root when present:
STREAM-style copy bandwidth and cuBLAS bf16 throughput).  The same cases are what the
committed ncu summaries under ``profiles/`` captured, e.g.::

    python -m myk_llm_b200.ops.kernel_cases gemm            # one case, timed
    python -m myk_llm_b200.ops.kernel_cases all             # every case, one JSON line each
    ncu --set full --clock-control none -k regex:gemm_kernel -s 1 -c 1 \\
        python -m myk_llm_b200.ops.kernel_cases gemm 3 --no-timing

Inputs exceed the 126 MB L2 wherever DRAM traffic is what the kernel is judged on.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"], "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def build(case: str):
    """(callable, flops per call, algorithmic bytes per call, description)."""
    from . import ext
    from . import flash_attn_func, fused_linear_cross_entropy, gemm, rms_norm

    torch.manual_seed(0)
    dev = "cuda"
    if case == "gemm":
        a = torch.randn(16384, 4096, device=dev).bfloat16()
        b = torch.randn(4096, 4096, device=dev).bfloat16()
        return (lambda: gemm(a, b)), 2 * 16384 * 4096 * 4096, (a.numel() + b.numel() + 16384 * 4096) * 2, \
            "bf16 GEMM 16384x4096x4096, bf16 out"
    if case == "gemm_fwd_200m":
        # the 200M model's gate/up projection: 32768 tokens x 1024 -> 5632, bf16 out
        x = torch.randn(32768, 1024, device=dev).bfloat16()
        w = torch.randn(5632, 1024, device=dev).bfloat16()
        return (lambda: gemm(x, w)), 2 * 32768 * 5632 * 1024, (x.numel() + w.numel() + 32768 * 5632) * 2, \
            "bf16 GEMM 32768x5632x1024 (200M gate/up forward), bf16 out"
    if case in ("gemm_gather_self_200m", "gemm_gather_prefetch_200m"):
        # the gate/up forward with the fused all-gather of a row-sharded weight, "ranks"
        # emulated as 8 buffers of this GPU: `self` gathers its own B operand (the producer
        # waits per 64 rows), `prefetch` gathers another weight while multiplying a held one
        world, n, k = 8, 5632, 1024
        x = torch.randn(32768, k, device=dev).bfloat16()
        w = torch.randn(n, k, device=dev).bfloat16()
        r = -(-n // world)
        shards = [torch.zeros(r * k, device=dev, dtype=torch.bfloat16) for _ in range(world)]
        for i, sh in enumerate(shards):
            part = w[i * r:(i + 1) * r].reshape(-1)
            sh[:part.numel()] = part
        ptrs = torch.tensor([sh.data_ptr() for sh in shards], dtype=torch.int64, device=dev)
        full = torch.empty_like(w)
        ready = torch.zeros((n + 63) // 64, dtype=torch.int32, device=dev)
        y = torch.empty(32768, n, device=dev, dtype=torch.bfloat16)
        held = w.clone()
        epoch = [0]

        def run():
            epoch[0] += 1
            b = full if case == "gemm_gather_self_200m" else held
            ext().gemm_gather(x, b, y, False, False, False, full, ptrs, 0, r, 3, ready, epoch[0])

        run.keep = shards  # the shards must outlive the closure
        return run, 2 * 32768 * n * k, (x.numel() + 2 * w.numel() + 32768 * n) * 2, \
            f"bf16 GEMM 32768x{n}x{k} with the fused gather of a {n}x{k} weight from {world} emulated ranks ({case})"
    if case == "gemm_wgrad_200m":
        # the 200M model's gate/up weight gradient: dW (5632 x 1024) += dy^T x over 32768 tokens
        dy = torch.randn(32768, 5632, device=dev).bfloat16()
        x = torch.randn(32768, 1024, device=dev).bfloat16()
        dw = torch.zeros(5632, 1024, device=dev)
        return (lambda: gemm(dy, x, a_major="mn", b_major="mn", out=dw, accumulate=True)), \
            2 * 32768 * 5632 * 1024, (dy.numel() + x.numel()) * 2 + dw.numel() * 8, \
            "bf16 GEMM wgrad 5632x1024x32768 (200M gate/up), fp32 accumulate (split-K reduce-add)"
    if case == "mxgemm":
        from . import mxfp8

        a = torch.randn(32768, 4096, device=dev).bfloat16()
        b = torch.randn(4096, 4096, device=dev).bfloat16()
        qa, sa = mxfp8.mx_quantize(a)
        qb, sb = mxfp8.mx_quantize(b)
        return (lambda: mxfp8.mx_gemm(qa, sa, "e4m3", qb, sb, "e4m3")), 2 * 32768 * 4096 * 4096, \
            qa.numel() + qb.numel() + 32768 * 4096 * 2, "MXFP8 GEMM 32768x4096x4096 (E4M3, 1x32 E8M0), bf16 out"
    if case == "mxquant":
        from . import mxfp8

        a = torch.randn(16384, 4096, device=dev).bfloat16()
        return (lambda: mxfp8.mx_quantize(a, "e4m3", True, True)), 0, a.numel() * (2 + 1 + 1), \
            "MXFP8 quantize 16384x4096 bf16 -> fp8 rows + fp8 transpose"
    if case in ("fp8quant_rows", "fp8quant_tensor", "fp8quant_cols_t"):
        # the 200M model's down-projection input (32768 tokens x 2816), 185 MB of bf16
        a = torch.randn(32768, 2816, device=dev).bfloat16()
        fn = {"fp8quant_rows": lambda: ext().fp8_quant_rows(a, False, True),
              "fp8quant_tensor": lambda: ext().fp8_quant_tensor(a, False),
              "fp8quant_cols_t": lambda: ext().fp8_quant_cols_t(a, False, True)}[case]
        return fn, 0, a.numel() * (2 + 1), f"float8 quantise ({case[9:]}) 32768x2816 bf16 -> e4m3"
    if case in ("fa_fwd", "fa_bwd"):
        q = torch.randn(4, 4096, 16, 128, device=dev).bfloat16().requires_grad_()
        k = torch.randn(4, 4096, 4, 128, device=dev).bfloat16().requires_grad_()
        v = torch.randn(4, 4096, 4, 128, device=dev).bfloat16().requires_grad_()
        attn = 4 * 16 * 4096 * 4096 / 2 * 128  # causal score entries x head_dim
        if case == "fa_fwd":
            return (lambda: flash_attn_func(q, k, v, causal=True)), 4 * attn, (q.numel() * 2 + k.numel() * 2) * 2, \
                "FlashAttention fwd B4 L4096 16q/4kv h128 causal"
        o = flash_attn_func(q, k, v, causal=True)
        do = torch.randn_like(o)
        return (lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True)), 10 * attn, \
            (q.numel() * 4 + k.numel() * 4) * 2, "FlashAttention bwd B4 L4096 16q/4kv h128 causal"
    if case in ("fa_fwd_h64", "fa_bwd_h64"):
        # the 200M model's attention: B8 L4096, 16 query / 4 KV heads of 64, causal
        q = torch.randn(8, 4096, 16, 64, device=dev).bfloat16().requires_grad_()
        k = torch.randn(8, 4096, 4, 64, device=dev).bfloat16().requires_grad_()
        v = torch.randn(8, 4096, 4, 64, device=dev).bfloat16().requires_grad_()
        attn = 8 * 16 * 4096 * 4096 / 2 * 64
        if case == "fa_fwd_h64":
            return (lambda: flash_attn_func(q, k, v, causal=True)), 4 * attn, (q.numel() * 2 + k.numel() * 2) * 2, \
                "FlashAttention fwd B8 L4096 16q/4kv h64 causal (200M layer)"
        o = flash_attn_func(q, k, v, causal=True)
        do = torch.randn_like(o)
        return (lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True)), 10 * attn, \
            (q.numel() * 4 + k.numel() * 4) * 2, "FlashAttention bwd B8 L4096 16q/4kv h64 causal (200M layer)"
    if case in ("fa_fwd_docs_h64", "fa_bwd_docs_h64"):
        # the 200M training step's attention: 8 rows of 4096 packed with the synthetic
        # loader's documents (geometric lengths, mean 1024), document-masked varlen
        import numpy as np

        from ..data.synthetic import packed_row
        from .attention import flash_attn_varlen_func

        lens = []
        for i in range(8):
            lens += packed_row(np.random.default_rng([0, i]), 4096, 65536, 1024, 0)["seqlens"].tolist()
        cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=dev)
        q = torch.randn(32768, 16, 64, device=dev).bfloat16().requires_grad_()
        k = torch.randn(32768, 4, 64, device=dev).bfloat16().requires_grad_()
        v = torch.randn(32768, 4, 64, device=dev).bfloat16().requires_grad_()
        attn = 16 * sum(n * n / 2 for n in lens) * 64

        def fwd():
            return flash_attn_varlen_func(q, k, v, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=4096,
                                          max_seqlen_k=4096, causal=True)

        what = f"FlashAttention {{}} 200M layer, 8x4096 packed with {len(lens)} synthetic documents, 16q/4kv h64"
        if case == "fa_fwd_docs_h64":
            return fwd, 4 * attn, (q.numel() * 2 + k.numel() * 2) * 2, what.format("fwd")
        o = fwd()
        do = torch.randn_like(o)
        return (lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True)), 10 * attn, \
            (q.numel() * 4 + k.numel() * 4) * 2, what.format("bwd")
    if case == "gdn":
        from .gdn import gated_delta_rule

        T, H = 16384, 16
        cu = torch.tensor([0, 1500, 1800, 5800, 6600, 9200, 10400, 11100, 14100, 15100, 16384], dtype=torch.int32,
                          device=dev)
        q, k, v = (torch.randn(1, T, H, 128, device=dev).bfloat16().requires_grad_() for _ in range(3))
        g = (-torch.rand(1, T, H, device=dev) * 0.2).requires_grad_()
        bt = torch.rand(1, T, H, device=dev).requires_grad_()
        o, _ = gated_delta_rule(q, k, v, g, bt, cu_seqlens=cu)
        do = torch.randn_like(o)
        return (lambda: torch.autograd.grad(o, (q, k, v, g, bt), do, retain_graph=True)), 0, \
            q.numel() * 2 * 8, "Gated DeltaNet backward T16384 (10 docs) H16 dk=dv=128"
    if case == "rmsnorm":
        x = torch.randn(32768, 2048, device=dev)
        w = torch.ones(2048, device=dev)
        return (lambda: rms_norm(x, w, 1e-6, out_dtype=torch.bfloat16)), 0, x.numel() * (4 + 2), \
            "RMSNorm fwd 32768x2048 fp32 in, bf16 out"
    if case == "ce":
        h = torch.randn(32768, 1024, device=dev).bfloat16()
        w = torch.randn(65536, 1024, device=dev) * 0.02
        t = torch.randint(0, 65536, (32768,), device=dev)
        return (lambda: fused_linear_cross_entropy(h, w, t, 32768.0, z_loss=1e-4)), 3 * 2 * 32768 * 65536 * 1024, \
            0, "fused linear + CE + z-loss fwd/bwd, 32768 tokens x vocab 65536 x 1024"
    if case == "decode_attn":
        q = torch.randn(64, 3, 16, 64, device=dev).bfloat16()
        kc = torch.randn(64, 2400, 4, 64, device=dev).bfloat16()
        vc = torch.randn_like(kc)
        lens = torch.full((64,), 2048, dtype=torch.int32, device=dev)
        return (lambda: ext().fa_decode(q, kc, vc, lens, 0.125, -1, 0)), 0, 64 * 2048 * 4 * 64 * 2 * 2, \
            "split-KV decode attention B64, 3 queries x 16q/4kv h64, 2048 cached keys"
    if case == "skinny":
        a = torch.randn(3, 2048, device=dev).bfloat16()
        w = torch.randn(65536, 2048, device=dev).bfloat16()
        y = torch.empty(3, 65536, device=dev, dtype=torch.bfloat16)
        return (lambda: ext().gemm_skinny(a, w, y)), 2 * 3 * 65536 * 2048, w.numel() * 2, \
            "skinny GEMM 3 x 2048 x 65536 (decode LM head)"
    raise ValueError(f"unknown case {case!r}")


CASES = ["gemm", "gemm_fwd_200m", "gemm_gather_self_200m", "gemm_gather_prefetch_200m", "gemm_wgrad_200m", "mxgemm", "mxquant", "fp8quant_rows", "fp8quant_tensor", "fp8quant_cols_t", "fa_fwd", "fa_bwd", "fa_fwd_h64", "fa_bwd_h64", "fa_fwd_docs_h64", "fa_bwd_docs_h64", "gdn", "rmsnorm", "ce", "decode_attn", "skinny"]


def time_case(case: str, reps: int = 20) -> dict:
    fn, flops, nbytes, desc = build(case)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    pk = _peaks()
    out = {"case": case, "what": desc, "ms": ms}
    if flops:
        out["tflops"] = flops / ms / 1e9
        out["frac_of_bf16_peak"] = out["tflops"] / pk["bf16_tflops"]
    if nbytes:
        out["gbs"] = nbytes / ms / 1e6
        out["frac_of_hbm"] = out["gbs"] / pk["hbm_gbs"]
    out["peaks"] = pk["source"]
    return out


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=CASES + ["all"])
    ap.add_argument("reps", nargs="?", type=int, default=20)
    ap.add_argument("--no-timing", action="store_true", help="just run the case reps times (for profilers)")
    args = ap.parse_args(argv)
    sys.path.insert(0, ROOT)
    for c in CASES if args.case == "all" else [args.case]:
        if args.no_timing:
            fn, *_ = build(c)
            for _ in range(args.reps):
                fn()
            torch.cuda.synchronize()
            print(json.dumps({"case": c, "ran": args.reps}))
        else:
            print(json.dumps(time_case(c, args.reps)), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
