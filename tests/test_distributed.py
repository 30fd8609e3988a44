"""Multi-process data parallelism on CPU (gloo, world size 2): the sharded runtime trains
exactly like one process on the whole global batch, for Muon + AdamW, in its three
layouts: row-sharded block weights gathered at every use (the FSDP2 default) or once per
step, and every parameter replicated with only optimizer state and work partitioned.  Also torch
FSDP2 (the NCCL-baseline strategy) over gloo on the tiny config, and the host-side
failure path: a rank that raises makes the other rank's next collective fail instead of
hanging."""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from myk_llm_b200.configuration import load_config
from myk_llm_b200.parallel.distributed import DistInfo
from myk_llm_b200.train.config import TrainConfig

OVERRIDES = ["model.num_layers=2", "data.seq_len=64", "data.micro_batch_size=2", "global_batch_size=4",
             "model.max_seq_len=64", "optimizer.name=muon", "optimizer.lr=3e-3", "optimizer.grad_clip=0.0", "optimizer.eps=1e-3",
             "schedule.kind=constant"]


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run_steps(trainer, world, rank, steps=3):
    from myk_llm_b200.data.synthetic import SyntheticLoader

    ld = SyntheticLoader(trainer.config.data, rank, world)
    for s in range(1, steps + 1):
        batches = [ld.batch_at((s - 1) * trainer.grad_accum + i) for i in range(trainer.grad_accum)]
        trainer.train_step(batches, s)
    full = getattr(trainer.model, "full_named_parameters", None)
    if full is not None:
        return full()
    return {n: p.detach().clone() for n, p in trainer.raw_model.named_parameters()}


def _worker(rank, world, port, out_path, strategy, reshard=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MYKB_PG_TIMEOUT_S="60")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml",
                      OVERRIDES + [f"parallel.strategy={strategy}", f"parallel.reshard_after_forward={str(reshard).lower()}"])
    tr = Trainer(cfg, DistInfo(rank, world, rank, torch.device("cpu")), build_data=False)
    params = _run_steps(tr, world, rank)
    if strategy == "fsdp":
        from torch.distributed.tensor import DTensor

        params = {n: (p.full_tensor() if isinstance(p, DTensor) else p) for n, p in params.items()}
    if rank == 0:
        torch.save(params, out_path)
    dist.barrier()
    dist.destroy_process_group()


def _single(tmp):
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OVERRIDES)
    tr = Trainer(cfg, DistInfo(0, 1, 0, torch.device("cpu")), build_data=False)
    return _run_steps(tr, 1, 0)


@pytest.mark.parametrize("strategy,reshard", [("sharded", True), ("sharded", False), ("replicated", False),
                                              ("fsdp", False)])
def test_world2_matches_single_process(strategy, reshard, tmp_path):
    out = str(tmp_path / "p.pt")
    mp.spawn(_worker, args=(2, _port(), out, strategy, reshard), nprocs=2, join=True)
    dp = torch.load(out)
    ref = _single(tmp_path)
    for n, p in ref.items():
        tol = 5e-4 if p.ndim == 2 and n.startswith("layers") else 1e-4  # bf16 Newton-Schulz noise
        assert torch.allclose(dp[n], p, atol=tol, rtol=1e-4), (n, (dp[n] - p).abs().max())


def _failing_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == 1:
        os._exit(3)  # a rank dies between steps
    try:
        dist.all_reduce(t)
        dist.all_reduce(t)
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_dead_rank_fails_fast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in ps)
    assert q.get(timeout=5) != "no error"


RESUME_OV = ["model.num_layers=2", "data.seq_len=64", "data.micro_batch_size=2", "global_batch_size=4",
             "model.max_seq_len=64", "optimizer.name=muon", "steps=6", "checkpoint.interval=2",
             "checkpoint.final=true", "checkpoint.keep_last=0", "logging.interval=1"]


def _fit_worker(rank, world, port, run_root, die_at, out_path):
    """Runs ``Trainer.fit`` as rank ``rank``; with ``die_at`` rank 1 exits abruptly when it
    reaches that step (between steps: nothing of its in flight)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", RESUME_OV + [f"output_dir={run_root}"])
    tr = Trainer(cfg, DistInfo(rank, world, rank, torch.device("cpu")))
    if die_at is not None and rank == 1:
        step_fn = tr.train_step

        def dying(batches, step=None):
            if step == die_at:
                os._exit(7)
            return step_fn(batches, step)

        tr.train_step = dying
    tr.fit("auto")
    full = tr.model.full_named_parameters() if hasattr(tr.model, "full_named_parameters") else \
        {n: p.detach().clone() for n, p in tr.raw_model.named_parameters()}
    if rank == 0 and out_path:
        torch.save(full, out_path)
    dist.barrier()
    dist.destroy_process_group()


def _run_fit(world, run_root, die_at=None, out_path=None):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_fit_worker, args=(r, world, port, str(run_root), die_at, out_path))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    return [p.exitcode for p in procs]


def test_killed_rank_fails_fast_and_the_job_resumes_bit_exactly(tmp_path):
    """A rank dies at step 5 (checkpoints at 2 and 4): every rank ends with an error rather
    than hanging; re-running the same command resumes from step 4 and ends with exactly the
    parameters of an uninterrupted run."""
    from myk_llm_b200.train.checkpoint import latest_checkpoint

    codes = _run_fit(2, tmp_path / "crashed", die_at=5)
    assert codes[1] == 7 and codes[0] != 0
    assert latest_checkpoint(tmp_path / "crashed" / "tiny-cpu").name == "step_0000004"
    assert _run_fit(2, tmp_path / "crashed", out_path=str(tmp_path / "resumed.pt")) == [0, 0]
    assert _run_fit(2, tmp_path / "clean", out_path=str(tmp_path / "clean.pt")) == [0, 0]
    resumed, clean = torch.load(tmp_path / "resumed.pt"), torch.load(tmp_path / "clean.pt")
    for name, p in clean.items():
        assert torch.equal(resumed[name], p), name


NGRAM = ["model.ngram.orders=[2,3]", "model.ngram.num_buckets=1031", "model.ngram.dim=256"]


def _ngram_worker(rank, world, port, out_path, ckpt):
    """World-2 training with row-sharded n-gram tables over gloo, a checkpoint after step 2,
    step 3, then the checkpoint loaded back and step 3 repeated."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MYKB_PG_TIMEOUT_S="60")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from myk_llm_b200.data.synthetic import SyntheticLoader
    from myk_llm_b200.train.checkpoint import load_checkpoint, save_checkpoint
    from myk_llm_b200.train.trainer import Trainer

    info = DistInfo(rank, world, rank, torch.device("cpu"))
    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OVERRIDES + NGRAM + ["parallel.strategy=sharded"])
    tr = Trainer(cfg, info, build_data=False)
    assert tr.model.tables is not None and tr.model.tables.rows_per_rank == 516
    ld = SyntheticLoader(tr.config.data, rank, world)

    def step(s):
        tr.train_step([ld.batch_at((s - 1) * tr.grad_accum + i) for i in range(tr.grad_accum)], s)

    step(1)
    step(2)
    save_checkpoint(ckpt, tr.model, tr.optimizers, {"step": 2}, None, info, export_weights=False)
    step(3)
    first = {n: p.clone() for n, p in tr.model.full_named_parameters().items()}
    load_checkpoint(ckpt, tr.model, tr.optimizers, info)
    step(3)
    again = tr.model.full_named_parameters()
    if rank == 0:
        torch.save({"first": first, "again": again}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_world2_row_sharded_ngram_tables_match_single_process_and_resume(tmp_path):
    """The hashed n-gram tables row-sharded over two gloo ranks (each rank holds about half
    of every table and its AdamW moments, and updates only its rows) train like one process
    holding the whole tables, and a DCP checkpoint of the sharded tables resumes exactly."""
    out = str(tmp_path / "p.pt")
    mp.spawn(_ngram_worker, args=(2, _port(), out, str(tmp_path / "ckpt")), nprocs=2, join=True)
    got = torch.load(out)
    from myk_llm_b200.train.trainer import Trainer

    cfg = load_config(TrainConfig, "configs/baseline/tiny_cpu.yaml", OVERRIDES + NGRAM)
    ref = _run_steps(Trainer(cfg, DistInfo(0, 1, 0, torch.device("cpu")), build_data=False), 1, 0)
    assert any("ngram" in n for n in ref)
    for n, p in ref.items():
        tol = 5e-4 if p.ndim == 2 and n.startswith("layers") else 1e-4  # bf16 Newton-Schulz noise
        assert torch.allclose(got["first"][n], p, atol=tol, rtol=1e-4), (n, (got["first"][n] - p).abs().max())
        assert torch.equal(got["again"][n], got["first"][n]), n
