"""Training-throughput benchmark: train tokens/s of the 200M dense pretraining config.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N

Model: d_model 1024, 24 layers of global GQA attention (16 query / 4 KV heads of 64, RoPE
theta 10000 on every layer), SwiGLU 2816, untied 65536 vocab, fused linear-CE with
z-loss 1e-4; Muon (5 Newton-Schulz steps) on 2-D block weights, AdamW elsewhere; random
init (std 0.02).  Data: synthetic packed documents (geometric lengths, mean 1024, capped
at 4096, uniform ids, EOS between documents), seq 4096, micro-batch 8 per GPU, one
micro-batch per GPU per step (weak scaling: global batch 8 x N), document-masked.

Timing: W untimed warm-up steps; then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the launching stream;
the reported time is the max over ranks.  A second loop of K steps measures the same
metric end to end through the public API (pinned host batches copied in every step, loss
read back to the host every step), by wall clock.  The working set (activations of
32K tokens, 400M parameters, optimizer state) is far above the 126 MB L2, so no L2 flush
is inserted.  nvidia-smi clocks are sampled during the timed loop.

``--impl reference`` runs the unmodified reference package installed under
``baseline/_ref`` through its own public API (MykLLM, parallelize with torch.compile and
FSDP2, build_optimizers, Objective) on the same config and data.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
BASELINE_TOKS = None  # the reference publishes no number for this metric and config on any GPU

_COMMON = ["objective.z_loss=1e-4", "optimizer.name=muon", "optimizer.muon_ns_steps=5"]

# name -> (config overrides, seq_len, micro-batch per GPU, description for the JSON line)
MODELS = {
    "200m": ([
        "model.vocab_size=65536", "model.hidden_size=1024", "model.num_layers=24", "model.layer_pattern=G",
        "model.max_seq_len=4096", "model.tie_embeddings=false", "model.norm_eps=1e-6",
        "model.attention.num_heads=16", "model.attention.num_kv_heads=4", "model.attention.head_dim=64",
        "model.attention.global_rope=all", "model.attention.rope_theta_global=10000.0",
        "model.ffn.multiplier=2.75", "model.ffn.multiple_of=256",
        "data.seq_len=4096", "data.micro_batch_size=8"] + _COMMON, 4096, 8,
        "200M dense (d1024 L24 16q/4kv h64, SwiGLU 2816, vocab 65536 untied)"),
    "1b-hybrid": ([
        "model.vocab_size=65536", "model.hidden_size=2048", "model.num_layers=24", "model.layer_pattern=DDDG",
        "model.max_seq_len=8192", "model.tie_embeddings=false", "model.norm_eps=1e-6",
        "model.attention.num_heads=16", "model.attention.num_kv_heads=4", "model.attention.head_dim=128",
        "model.attention.global_rope=all", "model.attention.rope_theta_global=10000.0",
        "model.deltanet.kind=gdn", "model.deltanet.num_heads=16", "model.deltanet.head_dim=128",
        "model.deltanet.expand_v=1.0", "model.deltanet.conv_size=4", "model.deltanet.use_short_conv=true",
        "model.deltanet.use_gate=true",
        "model.ngram.orders=[2,3]", "model.ngram.num_buckets=1048576", "model.ngram.dim=2048",
        "model.ffn.multiplier=2.75", "model.ffn.multiple_of=256",
        "data.seq_len=8192", "data.micro_batch_size=2"] + _COMMON, 8192, 2,
        "1B hybrid (d2048 L24 DDDG: 18 GDN 16x128 + 6 GQA 16q/4kv h128, SwiGLU 5632, 2/3-gram 2^20 x 2048, "
        "vocab 65536 untied)"),
    "1b-mxfp8": ([
        "model.vocab_size=65536", "model.hidden_size=2048", "model.num_layers=20", "model.layer_pattern=GL",
        "model.max_seq_len=4096", "model.tie_embeddings=false", "model.norm_eps=1e-6",
        "model.attention.num_heads=16", "model.attention.num_kv_heads=4", "model.attention.head_dim=128",
        "model.attention.sliding_window=1024", "model.attention.global_rope=all",
        "model.attention.rope_theta_global=10000.0", "model.ffn.multiplier=2.75", "model.ffn.multiple_of=256",
        "parallel.float8=mxfp8", "data.seq_len=4096", "data.micro_batch_size=4"] + _COMMON, 4096, 4,
        "1B dense MXFP8 (d2048 L20 GL, window 1024 on odd layers, 16q/4kv h128, SwiGLU 5632, vocab 65536 untied; "
        "all block linears MXFP8, E4M3 forward)"),
}


def _model_layers(model: str) -> int:
    for o in MODELS[model][0]:
        if o.startswith("model.num_layers="):
            return int(o.split("=", 1)[1])
    raise KeyError(model)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="200m", choices=sorted(MODELS), help="benchmark config (default: 200m)")
    ap.add_argument("--set", action="append", default=[], metavar="KEY=VALUE",
                    help="(experiments only) extra config overrides for our arm, e.g. parallel.float8=none")
    ap.add_argument("--layers", type=int, default=None,
                    help="(debug only) override the model's layer count; results are not comparable")
    ap.add_argument("--ref-compile", default="auto", choices=["auto", "on", "off"],
                    help="reference arm: its parallel.compile switch (auto: on, falling back to off if Inductor fails)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the timed loop runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        mhz, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ----------------------------------------------------------------------------- helpers
def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def synthetic_batches(n: int, step0: int, rank: int, world: int, batch_cls, seq_len: int, micro: int,
                      seed: int = 0):
    """The synthetic packed-document micro-batches of steps [step0, step0+n) for this rank,
    built on the host and pinned."""
    from myk_llm_b200.data.config import DataConfig, SyntheticDataConfig
    from myk_llm_b200.data.synthetic import SyntheticLoader

    # with several ranks, the global batch's rows go to ranks balanced by attention work
    # (the same global batch for both arms; only the row-to-rank mapping changes)
    cfg = DataConfig(kind="synthetic", seq_len=seq_len, micro_batch_size=micro, seed=seed,
                     synthetic=SyntheticDataConfig(vocab_size=65536, mean_doc_len=1024, eos_id=0,
                                                   balance_ranks=world > 1))
    ld = SyntheticLoader(cfg, rank, world)
    out = []
    for s in range(step0, step0 + n):
        b = ld.batch_at(s)
        out.append(batch_cls(b.input_ids.pin_memory(), b.targets.pin_memory(), b.seqlens))
    return out


def max_over_ranks(x: float, device) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, device) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier_sync(device):
    import torch
    import torch.distributed as dist

    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize(device)


def count_launches(step_fn, prefix: str) -> int:
    """Kernels whose name contains ``prefix`` launched by one step (profiled outside the
    timed region)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = 0
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA and prefix in e.name:
            n += 1
    return n


# ----------------------------------------------------------------------------- arms
def build_ours(world: int, layers: int, model: str, extra: list[str] | None = None):
    import torch

    from myk_llm_b200.configuration import apply_overrides, from_dict
    from myk_llm_b200.data.config import Batch
    from myk_llm_b200.parallel.distributed import init_distributed
    from myk_llm_b200.train.config import TrainConfig
    from myk_llm_b200.train.trainer import Trainer

    ov, _, micro, _ = MODELS[model]
    ov = ov + list(extra or []) + [f"global_batch_size={micro * world}", "steps=1000", "schedule.warmup_ratio=0.0",
                                   "data.kind=synthetic", "logging.tensorboard=false"]
    if layers is not None:
        ov.append(f"model.num_layers={layers}")
    cfg = from_dict(TrainConfig, apply_overrides({}, ov))
    info = init_distributed()
    tr = Trainer(cfg, info, build_data=False)
    state = {"step": 0}

    def step(batch):
        state["step"] += 1
        return tr.train_step([batch], state["step"])["loss"]

    return info.device, step, Batch, tr


def build_reference(world: int, layers: int, model: str, compile_blocks: bool = True):
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    import torch

    from myk_llm.configuration import apply_overrides, from_dict
    from myk_llm.data import Batch
    from myk_llm.model import MykLLM
    from myk_llm.train.config import TrainConfig
    from myk_llm.train.distributed import all_reduce_sum, init_distributed, parallelize
    from myk_llm.train.objectives import Objective
    from myk_llm.train.optim import build_optimizers

    ov, _, micro, _ = MODELS[model]
    ov = list(ov) + [f"global_batch_size={micro * world}", f"parallel.compile={'true' if compile_blocks else 'false'}"]
    if layers is not None:
        ov.append(f"model.num_layers={layers}")
    cfg = from_dict(TrainConfig, apply_overrides({}, ov))
    info = init_distributed()
    torch.manual_seed(cfg.seed)
    torch.set_float32_matmul_precision("high")
    model = parallelize(MykLLM(cfg.model).to(info.device), cfg.parallel, info)
    opts = build_optimizers(model, cfg.optimizer)
    obj = Objective(cfg.objective, info.device)
    params = [p for p in model.parameters() if p.requires_grad]

    def step(batch):
        b = batch.to(info.device)
        norm = all_reduce_sum(batch.num_targets, info.device)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(b.input_ids, seqlens=b.seqlens, head=obj.head(b, norm))
        out.loss.backward()
        torch.nn.utils.clip_grad_norm_(params, cfg.optimizer.grad_clip)
        for o in opts:
            o.step()
            o.zero_grad(set_to_none=True)
        return out.sums["ce"] / norm

    return info.device, step, Batch, None


def _parallel_desc(trainer, world: int) -> str:
    if world == 1 or trainer is None:
        return ""
    rt = trainer.model
    if getattr(rt, "shard_params", False):
        how = "re-gathered at every use" if rt.reshard_after_forward else "gathered once per step"
        return f" (block weights row-sharded, all-gather fused into the tcgen05 GEMMs, {how})"
    return " (parameters replicated, optimizer state sharded)"


def _compile_failure_reason(err: BaseException) -> str:
    """One line naming why Inductor could not build the reference's step.  The known case on
    this image (torch 2.11, Triton 3.6): Inductor re-emits the reference's own Triton
    FlashAttention kernel with the Python-float softmax scale typed fp64, so the scores, the
    running max / rescale factor and the rescaled accumulator become fp64, and Triton's
    ``tl.dot(p, v, acc)`` rejects an fp64 accumulator for an fp32 product."""
    text = f"{type(err).__name__}: {err}"
    if "tl.dot" in text or "_fwd_inner" in text or "acc * alpha" in text:
        return ("Inductor recompiles the reference's Triton FlashAttention with the float softmax scale typed fp64; "
                "the fp64 accumulator then fails tl.dot's accumulator-type check (Triton 3.6)")
    first = text.strip().splitlines()[0] if text.strip() else type(err).__name__
    return first[:300]


def main():
    a = parse()
    rank, world, local = dist_env()
    if a.gpus != world and world > 1:
        print(f"warning: --gpus {a.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    os.environ.setdefault("MYKB_PG_TIMEOUT_S", "600")
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    _, seq_len, micro, model_desc = MODELS[a.model]
    compile_on = None
    trainer = None
    if a.impl == "reference":
        ref_dir = os.path.join(ROOT, "baseline", "_ref", "myk_llm")
        if not os.path.isdir(ref_dir):
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
            return
        if a.model == "1b-mxfp8":
            try:
                import torchao  # noqa: F401  (the reference's MXFP8 path wraps torchao)
            except ImportError as err:
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable":
                                      f"the reference's MXFP8 linears need torchao, which is not installed ({err})"}))
                return
        if a.model == "1b-hybrid":
            try:
                import fla.modules.causal_conv1d  # noqa: F401  (the reference's Gated DeltaNet imports it)
            except ImportError as err:
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable":
                                      f"the reference's Gated DeltaNet needs fla.modules.causal_conv1d; the installed "
                                      f"flash-linear-attention has none ({err})"}))
                return
        compile_on = a.ref_compile in ("auto", "on")
        compile_error = None
        device, step, batch_cls, _ = build_reference(world, a.layers, a.model, compile_on)
        if a.ref_compile == "auto":
            # try one step with torch.compile; if Inductor cannot build the reference's
            # kernels on this GPU, rebuild the reference with its compile switch off
            probe = synthetic_batches(1, 10_000, rank, world, batch_cls, seq_len, micro)[0]
            ok = True
            try:
                step(probe)
            except Exception as err:  # noqa: BLE001
                ok = False
                compile_error = _compile_failure_reason(err)
                print(f"reference with torch.compile failed ({compile_error}); using parallel.compile=false",
                      file=sys.stderr)
            if dist.is_initialized():
                t = torch.tensor([1.0 if ok else 0.0], device=device)
                dist.all_reduce(t, op=dist.ReduceOp.MIN)
                ok = bool(t.item() > 0)
            if not ok:
                import torch._dynamo

                torch._dynamo.reset()
                compile_on = False
                device, step, batch_cls, _ = build_reference(world, a.layers, a.model, False)
    else:
        device, step, batch_cls, trainer = build_ours(world, a.layers, a.model, a.set)

    total_steps = a.warmup + a.steps + 1
    batches = synthetic_batches(total_steps, 0, rank, world, batch_cls, seq_len, micro)
    bi = iter(batches)
    for _ in range(a.warmup):
        step(next(bi))
    barrier_sync(device)
    launch_batch = next(bi)
    barrier_sync(device)

    # ---- device-timed loop
    clocks = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else local)
    clocks.start()
    time.sleep(0.3)
    timed = [next(bi) for _ in range(a.steps)]
    barrier_sync(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    last = None
    for b in timed:
        last = step(b)
    ev1.record()
    barrier_sync(device)
    clk = clocks.stop()
    dev_ms = ev0.elapsed_time(ev1)
    dev_ms = max_over_ranks(dev_ms, device)
    # each rank's step returns its share of the loss (local CE sum / global target count)
    loss_val = sum_over_ranks(float(last) if last is not None else float("nan"), device)

    # ---- end-to-end loop (public API, H2D + D2H every step).  It replays the timed loop's
    # host batches: packed documents of random lengths make the attention cost differ from
    # batch to batch, so the two loops must run the same batches to be comparable.
    e2e_batches = timed
    barrier_sync(device)
    t0 = time.perf_counter()
    for b in e2e_batches:
        float(step(b))
    barrier_sync(device)
    e2e_s = max_over_ranks(time.perf_counter() - t0, device)

    # kernel launches of this framework in one step (profiled after the timed loops)
    launches = 0
    if a.impl == "ours":
        launches = count_launches(lambda: step(launch_batch), "mykb") * a.steps
    barrier_sync(device)

    peak_gb = max_over_ranks(torch.cuda.max_memory_allocated(device) / 2 ** 30, device)
    mem_detail = None
    if trainer is not None and hasattr(trainer.model, "memory_bytes"):
        mem_detail = trainer.model.memory_bytes()
    tokens_per_step = micro * seq_len * world
    value = tokens_per_step * a.steps / (dev_ms / 1000.0)
    e2e = tokens_per_step * a.steps / e2e_s
    h2d = timed[0].input_ids.numel() * 8 * 2 + sum(x.numel() * 4 for x in (timed[0].seqlens or []))
    if rank == 0:
        rec = {
            "metric": "train tokens/sec at 1/2/4/8 B200 (200M, 1B hybrid); MTP decode tokens/sec",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": dev_ms / a.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None,
            "dtype": "mxfp8 (E4M3 operands, E8M0 1x32 scales; bf16 elsewhere)"
            if a.model == "1b-mxfp8" and "parallel.float8=none" not in a.set else "bf16",
            "data": "synthetic packed documents (geometric mean 1024, uniform ids, EOS), random-init weights",
            "config": {"model": model_desc,
                       "global_batch": micro * world, "seq_len": seq_len, "micro_batch_per_gpu": micro,
                       "parallelism": f"dp{world}" + _parallel_desc(trainer, world),
                       "optimizer": "Muon(ns=5)+AdamW", "z_loss": 1e-4,
                       "l2": "working set >> 126 MB L2 (no flush inserted)",
                       **({"row_assignment": "global batch rows balanced over ranks by attention work"}
                          if world > 1 else {}),
                       "layers": a.layers if a.layers is not None else _model_layers(a.model),
                       **({"overrides": a.set} if a.set else {})},
            "clocks": clk,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
            "gpu_launches": launches,
            "loss": loss_val,
            "peak_mem_gb_per_gpu": peak_gb,
        }
        if mem_detail:
            rec["config"]["memory_per_gpu_bytes"] = mem_detail
        if a.impl == "reference":
            rec["impl"] = "reference"
            rec["config"]["reference_compile"] = compile_on
            if compile_error:
                rec["config"]["reference_compile_error"] = compile_error
            rec.pop("gpu_launches")
        print(json.dumps(rec))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
