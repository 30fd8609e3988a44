"""The all-gather fused into the tcgen05 GEMM (``gemm_gather``) and the standalone gather
(``shard_gather``) against a plain fp32 PyTorch oracle.

On one GPU the "ranks" are separate buffers of that GPU: the kernel reads each rank's
shard through the pointer table whether it is a peer's memory or not, so this checks the
chunk bookkeeping, the row-to-owner arithmetic, the rotated tile / reduction order and
the counters across repeated calls.  On two GPUs the shards live in symmetric memory and
the comparison also includes NCCL's all-gather followed by the regular GEMM."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _close(got, ref, tol=2e-2):
    err = (got.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"err {err} > {tol} * {scale}"


def _shards(w: torch.Tensor, world: int):
    """Row shards of w padded to R rows each, in one flat buffer per rank."""
    rows, cols = w.shape
    r = -(-rows // world)
    bufs = []
    for i in range(world):
        b = torch.zeros(16 + r * cols, dtype=torch.bfloat16, device=w.device)  # 16 elements before the shard
        part = w[i * r:min(rows, (i + 1) * r)]
        b[16:16 + part.numel()] = part.reshape(-1)
        bufs.append(b)
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=w.device)
    return bufs, ptrs, r


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("m,n,k", [(512, 1536, 1024), (300, 1000, 520), (1024, 5632, 1024), (128, 64, 256)])
def test_gather_gemm_one_gpu_emulated_ranks(world, m, n, k):
    from myk_llm_b200.ops import ext

    if n < world:
        pytest.skip("fewer rows than ranks")
    g = torch.Generator(device="cuda").manual_seed(m + n + k + world)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16()
    bufs, ptrs, r = _shards(w, world)
    for rank in range(world):
        full = torch.empty(n, k, dtype=torch.bfloat16, device="cuda")
        ready = torch.zeros((n + 63) // 64, dtype=torch.int32, device="cuda")
        for epoch in (1, 2):  # twice: the counters carry over between calls
            x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
            y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
            full.fill_(float("nan"))  # every element must come from the shards
            ext().gemm_gather(x, full, y, False, False, False, full, ptrs, 16, r, rank, ready, epoch)
            torch.cuda.synchronize()
            assert ext().take_status() == 0
            assert torch.equal(full, w)
            _close(y, x.float() @ w.float().t())
        # data gradient: dx = dy W, the gather fused with a reduction over W's rows
        for epoch in (3, 4):
            dy = torch.randn(m, n, device="cuda", generator=g).bfloat16()
            dx = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
            full.fill_(float("nan"))
            ext().gemm_gather(dy, full, dx, False, True, False, full, ptrs, 16, r, rank, ready, epoch)
            torch.cuda.synchronize()
            assert ext().take_status() == 0
            assert torch.equal(full, w)
            _close(dx, dy.float() @ w.float())
        full.zero_()
        ext().shard_gather(full, ptrs, 16, r, rank, ready, 5)
        torch.cuda.synchronize()
        assert torch.equal(full, w)
    del bufs


@pytest.mark.parametrize("world", [2, 8])
def test_gather_as_prefetch_inside_unrelated_products(world):
    """The gather warps fill another weight's buffer while the GEMM multiplies operands
    that do not depend on it: forward, data-gradient and weight-gradient layouts."""
    from myk_llm_b200.ops import ext

    g = torch.Generator(device="cuda").manual_seed(world)
    w = (torch.randn(2816, 1024, device="cuda", generator=g) * 0.05).bfloat16()
    bufs, ptrs, r = _shards(w, world)
    full = torch.empty_like(w)
    ready = torch.zeros((w.shape[0] + 63) // 64, dtype=torch.int32, device="cuda")
    m, n, k = 2048, 1536, 1024
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16()
    epoch = 0
    for layout in ("fwd", "dgrad", "wgrad"):
        epoch += 1
        full.zero_()
        if layout == "fwd":
            d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
            ext().gemm_gather(x, b, d, False, False, False, full, ptrs, 16, r, 1 % world, ready, epoch)
            ref = x.float() @ b.float().t()
        elif layout == "dgrad":
            dy = torch.randn(m, n, device="cuda", generator=g).bfloat16()
            d = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
            ext().gemm_gather(dy, b, d, False, True, False, full, ptrs, 16, r, 1 % world, ready, epoch)
            ref = dy.float() @ b.float()
        else:
            dy = torch.randn(m, n, device="cuda", generator=g).bfloat16()
            d = torch.ones(n, k, dtype=torch.float32, device="cuda")
            ext().gemm_gather(dy, x, d, True, True, True, full, ptrs, 16, r, 1 % world, ready, epoch)
            ref = 1.0 + dy.float().t() @ x.float()
        torch.cuda.synchronize()
        assert ext().take_status() == 0
        assert torch.equal(full, w), layout
        _close(d, ref)
    del bufs


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    import torch.distributed._symmetric_memory as symm

    from myk_llm_b200.ops import ext, gemm

    res = {}
    for (m, n, k) in [(4096, 5632, 1024), (1000, 1536, 1024), (512, 1000, 520)]:
        g = torch.Generator(device=dev).manual_seed(n * k)  # same weight on every rank
        w = (torch.randn(n, k, device=dev, generator=g) * 0.05).bfloat16()
        r = -(-n // world)
        shard = symm.empty(r * k, dtype=torch.bfloat16, device=dev)
        shard.zero_()
        part = w[rank * r:min(n, (rank + 1) * r)]
        shard[:part.numel()] = part.reshape(-1)
        h = symm.rendezvous(shard, dist.group.WORLD)
        ptrs = torch.tensor(list(h.buffer_ptrs), dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        gx = torch.Generator(device=dev).manual_seed(1000 + rank)
        x = torch.randn(m, k, device=dev, generator=gx).bfloat16()
        full = torch.empty(n, k, dtype=torch.bfloat16, device=dev)
        ready = torch.zeros((n + 63) // 64, dtype=torch.int32, device=dev)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        ext().gemm_gather(x, full, y, False, False, False, full, ptrs, 0, r, rank, ready, 1)
        dy = torch.randn(m, n, device=dev, generator=gx).bfloat16()
        dx = torch.empty(m, k, dtype=torch.bfloat16, device=dev)
        full2 = torch.empty(n, k, dtype=torch.bfloat16, device=dev)
        ready2 = torch.zeros_like(ready)
        ext().gemm_gather(dy, full2, dx, False, True, False, full2, ptrs, 0, r, rank, ready2, 1)
        # the unfused baseline: NCCL all-gather of the padded shards, then the GEMM
        gathered = torch.empty(world * r * k, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(gathered, shard[:r * k].clone())
        wn = gathered.view(world * r, k)[:n]
        y_nccl = gemm(x, wn)
        torch.cuda.synchronize()
        status = int(ext().take_status())
        res[(m, n, k)] = dict(
            status=status, full_ok=bool(torch.equal(full, w)) and bool(torch.equal(full2, w)),
            y_vs_nccl=(y.float() - y_nccl.float()).abs().max().item(),
            y_err=(y.float() - x.float() @ w.float().t()).abs().max().item(),
            y_scale=(x.float() @ w.float().t()).abs().max().item(),
            dx_err=(dx.float() - dy.float() @ w.float()).abs().max().item(),
            dx_scale=(dy.float() @ w.float()).abs().max().item())
        dist.barrier()
        del h
    if rank == 0:
        torch.save(res, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gather_gemm_two_gpus_matches_nccl_and_fp32(tmp_path):
    out = str(tmp_path / "r.pt")
    mp.spawn(_worker, args=(2, _port(), out), nprocs=2, join=True)
    res = torch.load(out)
    for key, r in res.items():
        assert r["status"] == 0, key
        assert r["full_ok"], key
        assert r["y_vs_nccl"] == 0.0, (key, r)  # same operands, same kernel tiles: bit-identical
        assert r["y_err"] <= 2e-2 * r["y_scale"], (key, r)
        assert r["dx_err"] <= 2e-2 * r["dx_scale"], (key, r)
