"""MTP speculative-decode benchmark (random weights), one GPU or data-parallel replicas.

    python -m myk_llm_b200.infer.benchmark_decode                       # 200M + 2 MTP heads
    python -m myk_llm_b200.infer.benchmark_decode --batch 1 8 64 --prompt 2048 --new 256
    python -m myk_llm_b200.infer.benchmark_decode --impl reference      # the reference's own timing
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m myk_llm_b200.infer.benchmark_decode  # 8 replicas

With several ranks every GPU runs an independent replica (its own model copy, prompts
and decoder); rank 0 reports the sum of the replicas' tokens over the slowest replica's
time (prefill and decode timed separately, max over ranks).

Ours: :class:`~myk_llm_b200.infer.engine.StaticDecoder` prefills random prompts into
static KV caches, then decodes greedily with the model's MTP heads drafting K tokens per
round and the main model verifying them (one CUDA graph per round).  Prefill and decode
are timed with CUDA events; decode tokens/s counts the tokens emitted per row (trimmed to
``--new``) over the rounds that produced them, so it includes the real acceptance rate
(close to 0 with random weights, where every round yields ~1 token per row).

Reference arm: the reference's ``scripts/benchmark_decode.py`` times one captured verify +
draft iteration over static caches at a given context, for an assumed acceptance rate;
its tokens/s = batch * (1 + a + ... + a^K) / iteration time, evaluated here at the
acceptance our decoder measured, and its prefill is one forward pass of the prompts.
Each configuration prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

MODEL_OVERRIDES = [
    "vocab_size=65536", "hidden_size=1024", "num_layers=24", "layer_pattern=G", "tie_embeddings=false",
    "attention.num_heads=16", "attention.num_kv_heads=4", "attention.head_dim=64", "attention.global_rope=all",
    "attention.rope_theta_global=10000.0", "ffn.multiplier=2.75", "ffn.multiple_of=256", "mtp.depth=2",
]


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def bench_ours(batch: int, prompt: int, new: int, seed: int = 0) -> dict:
    from ..configuration import apply_overrides, from_dict
    from ..models import MykLLM, ModelConfig
    from .engine import StaticDecoder

    cfg = from_dict(ModelConfig, apply_overrides({}, MODEL_OVERRIDES + [f"max_seq_len={prompt + new + 8}"]))
    torch.manual_seed(seed)
    model = MykLLM(cfg).cuda().eval()  # fp32 masters; every op computes in bf16 (cached bf16 weights)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    prompts = torch.randint(0, cfg.vocab_size, (batch, prompt), device="cuda", generator=gen)
    dec = StaticDecoder(model, batch_size=batch, max_len=prompt + new + 4)
    dec.generate(prompts, 8, check_every=4)  # warm-up: kernels, graph capture
    torch.cuda.synchronize()
    # prefill alone
    e0, e1 = _events()
    e0.record()
    dec.prefill(prompts)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    # full generation: generate() prefills, captures one decode round as a CUDA graph (its
    # buffers are sized per call), then replays it until every row has `new` tokens, with a
    # host check every 8 rounds.  Decode time is the replay loop as the decoder measures it
    # (synchronised wall time); the capture is reported separately, like the reference's
    # benchmark, which times rounds of an already captured graph.
    e2, e3 = _events()
    e2.record()
    _, st = dec.generate(prompts, new, check_every=8)
    e3.record()
    torch.cuda.synchronize()
    total_ms = e2.elapsed_time(e3)
    decode_ms = max(st.decode_s * 1e3, 1e-6)
    capture_ms = max(total_ms - st.prefill_s * 1e3 - decode_ms, 0.0)
    return {"impl": "ours", "batch": batch, "prompt": prompt, "new_tokens": new, "draft_depth": dec.K,
            "prefill_ms": prefill_ms, "prefill_tokens_per_s": batch * prompt / (prefill_ms / 1e3),
            "decode_ms": decode_ms, "decode_tokens_per_s": batch * new / (decode_ms / 1e3),
            "graph_capture_ms": capture_ms, "generate_total_ms": total_ms,
            "rounds": st.rounds, "tokens_per_round": st.tokens_per_round, "acceptance": st.acceptance,
            "per_depth_accept": st.per_depth_accept}


def bench_reference(batch: int, prompt: int, new: int, acceptance: float, seed: int = 0) -> dict:
    """The reference's iteration timing (its scripts/benchmark_decode.py, run from
    baseline/_ref) at context = prompt, K = 2."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    script = os.path.join(ref, "ref_scripts", "benchmark_decode.py")
    if not os.path.exists(script):
        return {"impl": "reference", "unavailable": "baseline/_ref/ref_scripts/benchmark_decode.py is not installed"}
    sys.path.insert(0, ref)
    import importlib.util

    from myk_llm.configuration import apply_overrides, from_dict
    from myk_llm.model import MykLLM, ModelConfig

    spec = importlib.util.spec_from_file_location("ref_benchmark_decode", script)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # patches the reference's attention to static caches
    cfg = from_dict(ModelConfig, apply_overrides({}, MODEL_OVERRIDES + [f"max_seq_len={prompt + new + 8}"]))
    torch.manual_seed(seed)
    model = MykLLM(cfg).cuda().to(torch.bfloat16).eval()
    K = cfg.mtp.depth
    it_s = mod.iteration_time(model, batch, K, prompt, repeats=50)
    for m in model.modules():
        m.__dict__.pop("_static", None)
    ids = torch.randint(0, cfg.vocab_size, (batch, prompt), device="cuda")
    with torch.no_grad():
        model(ids)
        torch.cuda.synchronize()
        e0, e1 = _events()
        e0.record()
        model(ids)
        e1.record()
        torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    tokens_per_it = sum(acceptance ** i for i in range(K + 1))
    return {"impl": "reference", "batch": batch, "prompt": prompt, "new_tokens": new, "draft_depth": K,
            "prefill_ms": prefill_ms, "prefill_tokens_per_s": batch * prompt / (prefill_ms / 1e3),
            "iteration_ms": it_s * 1e3, "decode_tokens_per_s": batch * tokens_per_it / it_s,
            "acceptance_assumed": acceptance}


def _replicas(result: dict, world: int) -> dict:
    """Aggregate one replica per rank: times are the max over ranks, token rates the sum of
    the replicas' tokens over that time."""
    import torch.distributed as dist

    if world == 1 or "unavailable" in result:
        return result
    keys = [k for k in ("prefill_ms", "decode_ms", "iteration_ms") if k in result]
    t = torch.tensor([result[k] for k in keys], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out = dict(result, replicas=world)
    for k, v in zip(keys, t.tolist()):
        out[k] = v
    b, new, prompt = result["batch"], result["new_tokens"], result["prompt"]
    out["prefill_tokens_per_s"] = world * b * prompt / (out["prefill_ms"] / 1e3)
    if "decode_ms" in out:
        out["decode_tokens_per_s"] = world * b * new / (out["decode_ms"] / 1e3)
    else:
        tokens_per_it = sum(result["acceptance_assumed"] ** i for i in range(result["draft_depth"] + 1))
        out["decode_tokens_per_s"] = world * b * tokens_per_it / (out["iteration_ms"] / 1e3)
    return out


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--batch", type=int, nargs="+", default=[1, 8, 64])
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--new", type=int, default=256)
    ap.add_argument("--impl", choices=["ours", "reference", "both"], default="ours")
    args = ap.parse_args(argv)
    sys.path.insert(0, ROOT)
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", torch.cuda.current_device()))
    for b in args.batch:
        acc = 0.0
        if args.impl in ("ours", "both"):
            r = _replicas(bench_ours(b, args.prompt, args.new, seed=rank), world)
            acc = r["acceptance"]
            if rank == 0:
                print(json.dumps(r), flush=True)
        if args.impl in ("reference", "both"):
            r = _replicas(bench_reference(b, args.prompt, args.new, acc, seed=rank), world)
            if rank == 0:
                print(json.dumps(r), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
