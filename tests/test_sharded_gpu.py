"""The sharded data-parallel runtime on 2 GPUs trains like one GPU on the whole global
batch, in its three layouts: block weights row-sharded and gathered inside the GEMMs at
every use or once per step, and every parameter replicated (the peer-memory reduce-scatter
fused with the norm and the optimizer update in all three).  Skipped with fewer than 2
GPUs."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

OV = ["model.num_layers=2", "data.seq_len=256", "data.micro_batch_size=2", "global_batch_size=4",
      "model.max_seq_len=256", "optimizer.name=muon", "optimizer.lr=3e-3", "optimizer.grad_clip=0.0",
      "optimizer.eps=1e-3", "schedule.kind=constant"]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _steps(tr, world, rank, n=3):
    from myk_llm_b200.data.synthetic import SyntheticLoader

    ld = SyntheticLoader(tr.config.data, rank, world)
    for s in range(1, n + 1):
        tr.train_step([ld.batch_at((s - 1) * tr.grad_accum + i) for i in range(tr.grad_accum)], s)
    torch.cuda.synchronize()
    full = getattr(tr.model, "full_named_parameters", None)
    params = full() if full is not None else {k: v.detach() for k, v in tr.raw_model.named_parameters()}
    return {k: v.float().cpu().clone() for k, v in params.items()}


NGRAM = ["model.ngram.orders=[2,3]", "model.ngram.num_buckets=4099", "model.ngram.dim=256"]


def _worker(rank, world, port, out, strategy, reshard, nvls="0", extra=()):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MYKB_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0", MYKB_NVLS=nvls)
    from myk_llm_b200.configuration import load_config
    from myk_llm_b200.ops import ext
    from myk_llm_b200.parallel.distributed import init_distributed
    from myk_llm_b200.train.config import TrainConfig
    from myk_llm_b200.train.trainer import Trainer

    info = init_distributed()
    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml",
                      OV + list(extra) + [f"parallel.strategy={strategy}", f"parallel.reshard_after_forward={reshard}"])
    tr = Trainer(cfg, info, build_data=False)
    params = _steps(tr, world, rank)
    status = ext().take_status()
    if rank == 0:
        torch.save({"params": params, "status": status}, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("strategy,reshard,nvls", [("sharded", "true", "0"), ("sharded", "false", "0"),
                                                   ("replicated", "false", "0"), ("sharded", "true", "1")])
def test_sharded_two_gpus_matches_one(strategy, reshard, nvls, tmp_path):
    """nvls=1: the gradient reduce-scatter reads through NVSwitch multicast where the GPUs
    support it (peer loads otherwise)."""
    out = str(tmp_path / "p.pt")
    mp.spawn(_worker, args=(2, _port(), out, strategy, reshard, nvls), nprocs=2, join=True)
    got = torch.load(out)
    assert got["status"] == 0
    from myk_llm_b200.configuration import load_config
    from myk_llm_b200.parallel.distributed import DistInfo
    from myk_llm_b200.train.config import TrainConfig
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OV)
    tr = Trainer(cfg, DistInfo(0, 1, 0, torch.device("cuda", 0)), build_data=False)
    ref = _steps(tr, 1, 0)
    for n, p in ref.items():
        d = (got["params"][n] - p).abs().max().item()
        assert d < 3e-3, (n, d)


def _ngram_worker(rank, world, port, out, ckpt):
    """Three steps with row-sharded n-gram tables, a checkpoint, a fourth step; then the
    checkpoint is loaded back and the fourth step repeated: it must give the same values."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MYKB_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0", MYKB_NVLS="0")
    from myk_llm_b200.configuration import load_config
    from myk_llm_b200.data.synthetic import SyntheticLoader
    from myk_llm_b200.ops import ext
    from myk_llm_b200.parallel.distributed import init_distributed
    from myk_llm_b200.train.checkpoint import load_checkpoint, save_checkpoint
    from myk_llm_b200.train.config import TrainConfig
    from myk_llm_b200.train.trainer import Trainer

    info = init_distributed()
    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OV + NGRAM + ["parallel.strategy=sharded"])
    tr = Trainer(cfg, info, build_data=False)
    assert tr.model.tables is not None, "the n-gram tables should be row-sharded"
    params3 = _steps(tr, world, rank, n=3)
    save_checkpoint(ckpt, tr.model, tr.optimizers, {"step": 3}, None, info, export_weights=False)
    ld = SyntheticLoader(tr.config.data, rank, world)
    step4 = [ld.batch_at(3 * tr.grad_accum + i) for i in range(tr.grad_accum)]
    tr.train_step(step4, 4)
    first = {k: v.float().cpu().clone() for k, v in tr.model.full_named_parameters().items()}
    load_checkpoint(ckpt, tr.model, tr.optimizers, info)
    back = {k: v.float().cpu().clone() for k, v in tr.model.full_named_parameters().items()}
    tr.train_step(step4, 4)
    again = {k: v.float().cpu().clone() for k, v in tr.model.full_named_parameters().items()}
    status = ext().take_status()
    mem = tr.model.memory_bytes()["ngram_table_shards"]
    if rank == 0:
        torch.save({"params": params3, "back": back, "first": first, "again": again, "status": status, "mem": mem}, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_row_sharded_ngram_tables_match_one_gpu_and_resume(tmp_path):
    """n-gram tables row-sharded over 2 GPUs (peer row reads, peer gradient reductions,
    AdamW on the owned rows) train like one GPU with the whole tables, and a DCP checkpoint
    of the sharded tables and their moments resumes exactly."""
    out = str(tmp_path / "p.pt")
    mp.spawn(_ngram_worker, args=(2, _port(), out, str(tmp_path / "ckpt")), nprocs=2, join=True)
    got = torch.load(out)
    assert got["status"] == 0
    buckets, dim, orders = 4099, 256, 2
    assert got["mem"] == 4 * 4 * orders * ((-(-buckets // 2) * dim + 15) // 16 * 16)
    from myk_llm_b200.configuration import load_config
    from myk_llm_b200.parallel.distributed import DistInfo
    from myk_llm_b200.train.config import TrainConfig
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OV + NGRAM)
    tr = Trainer(cfg, DistInfo(0, 1, 0, torch.device("cuda", 0)), build_data=False)
    ref = _steps(tr, 1, 0)
    assert any("ngram" in n for n in ref)
    for n, p in ref.items():
        d = (got["params"][n] - p).abs().max().item()
        assert d < 3e-3, (n, d)
    for n, p in got["params"].items():
        assert torch.equal(got["back"][n], p), n  # the checkpoint restored step 3 exactly
        # and step 4 repeats (up to the order of the gradient reductions into table rows)
        assert (got["again"][n] - got["first"][n]).abs().max().item() < 1e-5, n


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_mxfp8_weights_gathered_in_fp8_match_one_gpu(tmp_path):
    """MXFP8 linears row-sharded over 2 GPUs: each rank quantises its own rows and the
    GEMMs read the fp8 values and E8M0 scales gathered from both ranks (one rank owns all
    128 rows of the 128-row weights, the other none); training matches one GPU with the
    same recipe."""
    extra = ["parallel.float8=mxfp8"]
    out = str(tmp_path / "p.pt")
    mp.spawn(_worker, args=(2, _port(), out, "sharded", "true", "0", extra), nprocs=2, join=True)
    got = torch.load(out)
    assert got["status"] == 0
    from myk_llm_b200.configuration import load_config
    from myk_llm_b200.parallel.distributed import DistInfo
    from myk_llm_b200.train.config import TrainConfig
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OV + extra)
    tr = Trainer(cfg, DistInfo(0, 1, 0, torch.device("cuda", 0)), build_data=False)
    ref = _steps(tr, 1, 0)
    for n, p in ref.items():
        d = (got["params"][n] - p).abs().max().item()
        assert d < 5e-3, (n, d)
