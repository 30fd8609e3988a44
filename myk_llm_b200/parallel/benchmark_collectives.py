"""Timing of the fused compute + collective kernels on real peers (one process per GPU).

    torchrun --nproc-per-node N -m myk_llm_b200.parallel.benchmark_collectives [--reps 20]

Cases, on the 200M model's shapes (max over ranks of CUDA-event times, after warm-up):

* ``gemm``             the gate/up forward GEMM x (32768 x 1024) W^T with W (5632 x 1024)
                       local: the compute reference;
* ``gemm_gather_self`` the same product with W row-sharded over the ranks in symmetric
                       memory: the GEMM's gather warps copy the other ranks' rows over
                       NVLink (16-byte peer loads) into a local buffer and the TMA producer
                       waits per 64 rows (the first use of a weight in a step);
* ``gemm_gather_next`` the product on a weight already held while the gather warps fetch
                       the next weight (the prefetch form the runtime uses);
* ``reduce_sumsq``     the gradient reduce-scatter fused with the clipping norm on a
                       403M-element fp32 buffer (the 200M model's parameters): every rank
                       sums its 1/N slice from every rank's buffer with peer loads;
* ``reduce_sumsq_nvls`` the same through NVSwitch multicast (``multimem.ld_reduce``) when
                       the GPUs support it.

Each line reports the roofline of the case: the slower of the FLOPs at the measured
bf16 peak (``MEASURED_PEAKS.json``) and the bytes that must cross NVLink per rank at the
measured 770 GB/s per direction, and the achieved fraction of it.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200s


def _peaks() -> dict:
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def _time(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main() -> None:
    import torch.distributed._symmetric_memory as symm

    from ..ops import ext, gemm
    from .distributed import init_distributed

    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    info = init_distributed()
    rank, world, dev = info.rank, info.world_size, info.device
    peaks = _peaks()
    e = ext()
    out = []

    def report(case: str, ms: float, flops: float, nvlink_bytes: float, note: str) -> None:
        t_flops = flops / (peaks["bf16_tflops"] * 1e12) * 1e3 if flops else 0.0
        t_link = nvlink_bytes / (NVLINK_GBS * 1e9) * 1e3
        roof = max(t_flops, t_link)
        out.append({"case": case, "world": world, "ms": round(ms, 4),
                    "tflops": round(flops / ms / 1e9, 1) if flops else None,
                    "nvlink_gb_per_rank": round(nvlink_bytes / 1e9, 4), "roofline_ms": round(roof, 4),
                    "frac_of_roofline": round(roof / ms, 3), "bound": "compute" if t_flops >= t_link else "nvlink",
                    "what": note})

    # ---- all-gather fused into the GEMM (gate/up forward of the 200M model)
    m, n, k = 32768, 5632, 1024
    torch.manual_seed(0)
    x = torch.randn(m, k, device=dev).bfloat16()
    w = torch.randn(n, k, device=dev).bfloat16()
    r = -(-n // world)
    shard = symm.empty(r * k, dtype=torch.bfloat16, device=dev)
    shard.zero_()
    part = w[rank * r:min(n, (rank + 1) * r)].reshape(-1)
    shard[:part.numel()].copy_(part)
    handle = symm.rendezvous(shard, dist.group.WORLD)
    ptrs = torch.tensor(list(handle.buffer_ptrs), dtype=torch.int64, device=dev)
    full = torch.empty_like(w)
    ready = torch.zeros((n + 63) // 64, dtype=torch.int32, device=dev)
    y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    held = w.clone()
    epoch = [0]
    torch.cuda.synchronize()
    dist.barrier()

    def gathered(b: torch.Tensor):
        def run():
            epoch[0] += 1
            e.gemm_gather(x, b, y, False, False, False, full, ptrs, 0, r, rank, ready, epoch[0])
        return run

    flops = 2.0 * m * n * k
    remote = (n - r) * k * 2 if world > 1 else 0
    report("gemm", _time(lambda: gemm(x, held, out=y), a.reps), flops, 0.0, f"bf16 {m}x{n}x{k}, W local")
    ms = _time(gathered(full), a.reps)
    if rank == 0:
        ok = torch.equal(full, w)
    report("gemm_gather_self", ms, flops, remote, "W row-sharded; the GEMM gathers its own W over NVLink")
    report("gemm_gather_next", _time(gathered(held), a.reps), flops, remote,
           "W held; the gather warps fetch another row-sharded weight during the product")

    # ---- reduce-scatter fused with the clipping norm (200M parameter count)
    numel = 403_000_000 // (16 * world) * 16 * world
    grad = symm.empty(numel, dtype=torch.float32, device=dev)
    grad.fill_(1.0 + rank)
    gh = symm.rendezvous(grad, dist.group.WORLD)
    gptrs = torch.tensor(list(gh.buffer_ptrs), dtype=torch.int64, device=dev)
    per = numel // world
    offsets = torch.tensor([rank * per], dtype=torch.int64, device=dev)
    prefix = torch.tensor([0, per], dtype=torch.int64, device=dev)
    partial = torch.zeros(1, device=dev)
    link = (world - 1) * per * 4.0  # each rank reads its slice from every other rank
    torch.cuda.synchronize()
    dist.barrier()
    report("reduce_sumsq", _time(lambda: e.dp_reduce_sumsq(gptrs, rank, world, offsets, prefix, partial, per),
                                 a.reps), 0.0, link, f"{numel / 1e6:.0f}M fp32, peer loads")
    from torch._C._autograd import DeviceType
    from torch._C._distributed_c10d import _SymmetricMemory

    mc_ok = torch.tensor([1 if _SymmetricMemory.has_multicast_support(DeviceType.CUDA, dev.index) else 0], device=dev)
    dist.all_reduce(mc_ok, op=dist.ReduceOp.MIN)
    if int(mc_ok) and world > 1:
        mc = int(gh.multicast_ptr) + (grad.data_ptr() - int(gh.buffer_ptrs[rank]))
        report("reduce_sumsq_nvls", _time(lambda: e.dp_reduce_sumsq_multimem(mc, grad, offsets, prefix, partial, per),
                                          a.reps), 0.0, (world - 1) * per * 4.0,
               f"{numel / 1e6:.0f}M fp32, NVSwitch multicast reduction")
    if rank == 0:
        for line in out:
            print(json.dumps(line))
        print(json.dumps({"gather_result_exact": bool(ok)}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
