"""Process groups and the choice of data-parallel runtime.

``init_distributed`` reads torchrun's environment (RANK, WORLD_SIZE, LOCAL_RANK,
MASTER_ADDR/PORT); without RANK it runs single-process.  On CUDA the group is NCCL, on
CPU gloo (tests).  The timeout is short by default so that ranks that lose a peer end
with an error instead of waiting for good (``MYKB_PG_TIMEOUT_S`` overrides it).

``parallelize`` applies, in order: MXFP8 conversion, activation checkpointing, then the
data-parallel runtime:

* ``fsdp``: torch FSDP2 (``fully_shard`` per block + root, fp32 gradient reduction as a
  sum, as in the reference ``src/myk_llm/train/distributed.py:108-134``): the NCCL
  baseline.
* ``sharded`` (and ``auto`` with more than one rank): this framework's parameter-sharded
  data parallel (:mod:`myk_llm_b200.parallel.sharded`): block weights row-sharded over the
  ranks and gathered inside the GEMMs that consume them, the gradient reduce-scatter fused
  with the clipping norm and the optimizer update, all over peer memory;
* ``replicated``: the same runtime with every parameter replicated (optimizer state and
  work still sharded).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.nn as nn


@dataclass
class DistInfo:
    rank: int
    world_size: int
    local_rank: int
    device: torch.device

    @property
    def is_main(self) -> bool:
        return self.rank == 0

    @property
    def enabled(self) -> bool:
        return self.world_size > 1


def init_distributed(device_type: str | None = None, timeout_s: float | None = None) -> DistInfo:
    use_cuda = torch.cuda.is_available() if device_type is None else device_type == "cuda"
    timeout = timedelta(seconds=float(os.environ.get("MYKB_PG_TIMEOUT_S", timeout_s or 600)))
    if "RANK" not in os.environ:
        if use_cuda:
            torch.cuda.set_device(0)
            return DistInfo(0, 1, 0, torch.device("cuda", 0))
        return DistInfo(0, 1, 0, torch.device("cpu"))
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ.get("LOCAL_RANK", 0))
    if use_cuda:
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        if not dist.is_initialized():
            dist.init_process_group("nccl", timeout=timeout, device_id=device)
            _host_group(timeout)
    else:
        device = torch.device("cpu")
        if not dist.is_initialized():
            dist.init_process_group("gloo", timeout=timeout)
    return DistInfo(rank, world, local, device)


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


_HOST_GROUP: list = []


def _host_group(timeout: timedelta | None = None):
    """A gloo group over the same ranks for host-side scalars (created once, by every rank
    at the same point, right after the NCCL group); the default group when it is gloo."""
    if not _HOST_GROUP:
        if dist.get_backend() == "gloo":
            _HOST_GROUP.append(dist.group.WORLD)
        else:
            kw = {"timeout": timeout} if timeout is not None else {}
            _HOST_GROUP.append(dist.new_group(backend="gloo", **kw))
    return _HOST_GROUP[0]


def all_reduce_sum(value: float | int, device: torch.device) -> float:  # noqa: ARG001
    """Sum of a host value over the ranks, on the host (gloo).  A per-step scalar such as the
    global target count then costs no GPU work and no device synchronisation, so each
    rank's host keeps queueing the next step's kernels while its GPU still runs this one."""
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, group=_host_group())
    return float(t[0])


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def uses_fsdp(config, info: DistInfo) -> bool:
    return config.strategy == "fsdp"


def uses_sharded(config, info: DistInfo) -> bool:
    return config.strategy in ("sharded", "replicated") or (config.strategy == "auto" and info.enabled)


def convert_float8(model: nn.Module, recipe: str, *, skip_down_proj: bool = False, grad_dtype: str = "e4m3") -> int:
    """Swap eligible block linears for float8 training modules; returns the count.  Skips
    the output head, DeltaNet a/b/f projections, optionally ``down_proj`` and linears
    whose dimensions are not multiples of 32 (MXFP8) or 16 (per-tensor / per-row float8)
    (reference selection rules, ``src/myk_llm/train/distributed.py:71-105``).  ``mxfp8``
    uses the block-scaled tcgen05 GEMMs; ``tensorwise``, ``rowwise`` and
    ``rowwise_with_gw_hp`` the dynamic-scaling linears of ``ops.float8``."""
    from ..ops import float8 as f8

    if recipe != "mxfp8" and recipe not in f8.RECIPES:
        raise ValueError(f"unknown float8 recipe {recipe!r}")
    align = 32 if recipe == "mxfp8" else 16

    def eligible(m: nn.Module, fqn: str) -> bool:
        return (type(m) is nn.Linear and fqn != "lm_head" and not fqn.endswith((".a_proj", ".b_proj"))
                and ".f_proj." not in fqn and not (skip_down_proj and fqn.endswith(".down_proj"))
                and m.in_features % align == 0 and m.out_features % align == 0)

    if recipe == "mxfp8":
        from ..ops.mxfp8 import convert_to_mxfp8_training

        return convert_to_mxfp8_training(model, module_filter_fn=eligible, grad_dtype=grad_dtype)
    return f8.convert_to_float8_training(model, recipe, module_filter_fn=eligible)


def parallelize(model, config, info: DistInfo):
    if config.float8 != "none":
        convert_float8(model, config.float8, skip_down_proj=config.float8_skip_down_proj,
                       grad_dtype=getattr(config, "mxfp8_grad_dtype", "e4m3"))
    if config.activation_checkpointing:
        model.set_activation_checkpointing(config.activation_checkpointing)
    if uses_fsdp(config, info):
        from torch.distributed.fsdp import FSDPModule, MixedPrecisionPolicy, fully_shard

        policy = MixedPrecisionPolicy(param_dtype=torch.bfloat16 if config.param_dtype == "bf16" else None,
                                      reduce_dtype=torch.float32)
        for block in model.blocks:
            fully_shard(block, mp_policy=policy, reshard_after_forward=config.reshard_after_forward)
        fully_shard(model, mp_policy=policy, reshard_after_forward=config.reshard_after_forward)
        gloo = dist.get_backend() == "gloo"
        for m in model.modules():
            if isinstance(m, FSDPModule):
                m.set_gradient_divide_factor(1.0)
                if gloo:  # gloo has no PREMUL_SUM: plain SUM (the factor is 1 anyway)
                    m.set_force_sum_reduction_for_comms(True)
        return model
    if uses_sharded(config, info) and info.enabled:
        from .sharded import shard_model

        return shard_model(model, info, reshard_after_forward=config.reshard_after_forward,
                           shard_params=config.strategy != "replicated")
    return model
