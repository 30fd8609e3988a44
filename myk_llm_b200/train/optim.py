"""Optimizers (Muon + AdamW) and learning-rate schedules.

Semantics, parameter-group keys and optimizer-state keys match the reference
(``src/myk_llm/train/optim.py:17-284``): ``Muon`` keeps ``momentum_buffer`` per
parameter and the group keys (lr, weight_decay, momentum, nesterov, ns_steps, adjust_lr);
AdamW is ``torch.optim.AdamW``'s state layout (step, exp_avg, exp_avg_sq) so DCP
checkpoints interchange.  The arithmetic runs on this framework's kernels:

* AdamW: one multi-tensor kernel launch per parameter group.
* Muon, local CUDA parameters: parameters are bucketed by shape; one kernel does the
  momentum lerp, Nesterov blend and bf16 pack of a whole bucket, Newton-Schulz runs as
  batched tcgen05 GEMMs on the bucket, one kernel applies decay + update.
* Muon under torch FSDP2 (DTensor shards, the NCCL baseline): the reference's
  owner-sharded scheme (bf16 all-to-all so each rank orthogonalises 1/world of the
  matrices).
* Muon under this framework's sharded runtime: the runtime supplies a fused
  gather / Newton-Schulz / scatter (``myk_llm_b200.parallel``).
"""

from __future__ import annotations

import math
from collections import defaultdict
from dataclasses import dataclass
from typing import Callable, Literal

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops
from ..ops.reference import newton_schulz_ref
from .config import OptimizerConfig, ScheduleConfig

NS_COEFFICIENTS = (3.4445, -4.7750, 2.0315)


def newton_schulz_orthogonalize(grad: torch.Tensor, steps: int, eps: float = 1e-7) -> torch.Tensor:
    """U V^T approximation of one matrix (bf16 quintic Newton-Schulz)."""
    if grad.is_cuda:
        return ops.batched_newton_schulz_orthogonalize(grad[None], steps, eps=eps)[0]
    return newton_schulz_ref(grad, steps, eps)


def lr_ratio(shape, mode: str) -> float:
    rows, cols = shape[0], shape[1]
    if mode == "original":
        return math.sqrt(max(1.0, rows / cols))
    if mode == "match_rms_adamw":
        return 0.2 * math.sqrt(max(rows, cols))
    return 1.0


def _is_dtensor(t: torch.Tensor) -> bool:
    try:
        from torch.distributed.tensor import DTensor

        return isinstance(t, DTensor)
    except ImportError:  # pragma: no cover
        return False


class Muon(torch.optim.Optimizer):
    """Momentum + orthogonalised updates for 2-D weights (see module docstring)."""

    def __init__(self, params, lr: float, weight_decay: float, momentum: float = 0.95, nesterov: bool = True,
                 ns_steps: int = 5, adjust_lr: Literal["original", "match_rms_adamw", "none"] = "match_rms_adamw"):
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                        adjust_lr=adjust_lr)
        super().__init__(params, defaults)
        # Set by the sharded runtime: fn(items, group) performs the whole update for
        # parameters it owns (items: list of (param, grad, momentum_buffer)).
        self.sharded_step: Callable | None = None
        # Optional one-element device tensor multiplying every gradient of the next step
        # (the clipping coefficient); the CUDA kernels apply it as they read the gradient.
        self.grad_scale: torch.Tensor | None = None

    _lr_ratio = staticmethod(lr_ratio)

    @torch.no_grad()
    def step(self, closure=None):  # type: ignore[override]
        for group in self.param_groups:
            lr, wd, mu = group["lr"], group["weight_decay"], group["momentum"]
            nesterov, ns_steps, mode = group["nesterov"], group["ns_steps"], group["adjust_lr"]
            local: dict[tuple, list] = defaultdict(list)
            fsdp: dict[tuple, list] = defaultdict(list)
            sharded, slow = [], []
            for p in group["params"]:
                g = p.grad
                if g is None:
                    continue
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32) if not _is_dtensor(p) \
                        else torch.zeros_like(g)
                buf = st["momentum_buffer"]
                if getattr(p, "_mykb_sharded", False) and self.sharded_step is not None:
                    sharded.append((p, g, buf))
                elif _is_dtensor(p):
                    fsdp[(tuple(p.shape), p.dtype)].append((p, g, buf))
                elif p.ndim == 2 and p.dtype == torch.float32 and p.is_contiguous() and g.is_contiguous():
                    local[(tuple(p.shape), g.dtype, p.device)].append((p, g, buf))
                else:
                    slow.append((p, g, buf))
            scale = self.grad_scale
            if scale is not None:  # paths without a scaling kernel scale their gradients first
                rest = [g for its in fsdp.values() for _, g, _ in its] + [g for _, g, _ in sharded + slow]
                if rest:
                    torch._foreach_mul_(rest, scale)
            for items in local.values():
                self._step_local_bucket(items, lr, wd, mu, nesterov, ns_steps, mode, scale)
            for items in fsdp.values():
                self._step_fsdp_bucket(items, lr, wd, mu, nesterov, ns_steps, mode)
            if sharded:
                self.sharded_step(sharded, group)
            for p, g, buf in slow:
                buf.lerp_(g.to(buf.dtype), 1 - mu)
                u = g.to(buf.dtype).lerp(buf, mu) if nesterov else buf
                if _is_dtensor(u):
                    from torch.distributed.tensor import distribute_tensor

                    full = newton_schulz_ref(u.full_tensor(), ns_steps)
                    u = distribute_tensor(full, u.device_mesh, u.placements, src_data_rank=None)
                else:
                    u = newton_schulz_orthogonalize(u, ns_steps)
                p.mul_(1 - lr * wd)
                p.add_(u.to(p.dtype), alpha=-lr * lr_ratio(p.shape, mode))

    @staticmethod
    def _step_local_bucket(items, lr, wd, mu, nesterov, ns_steps, mode, grad_scale=None):
        params = [p for p, _, _ in items]
        rows, cols = params[0].shape
        packed = torch.empty(len(items), rows, cols, dtype=torch.bfloat16, device=params[0].device)
        ops.muon_prepare([g for _, g, _ in items], [b for _, _, b in items], mu, nesterov, packed, grad_scale)
        orth = ops.batched_newton_schulz_orthogonalize(packed, ns_steps)
        ops.muon_apply(params, orth, lr, wd, -lr * lr_ratio((rows, cols), mode))

    @staticmethod
    def _step_fsdp_bucket(items, lr, wd, mu, nesterov, ns_steps, mode):
        """Owner-sharded Muon over torch FSDP2 DTensor shards (bf16 all-to-all)."""
        p0 = items[0][0]
        rows, cols = p0.shape
        mesh = p0.device_mesh
        world = mesh.size()
        shard_rows = rows // world
        lp = [p.to_local() for p, _, _ in items]
        lg = [g.to_local() for _, g, _ in items]
        lb = [b.to_local() for _, _, b in items]
        torch._foreach_lerp_(lb, lg, 1.0 - mu)
        upd = torch._foreach_lerp(lg, lb, mu) if nesterov else lb
        if world == 1 or rows % world:
            if world == 1:
                packed = torch.stack([u.bfloat16() for u in upd])
                orth = ops.batched_newton_schulz_orthogonalize(packed, ns_steps) if packed.is_cuda else \
                    newton_schulz_ref(packed, ns_steps)
                shards = list(orth)
            else:
                from torch.distributed.tensor import DTensor, distribute_tensor

                shards = []
                for (p, _, _), u in zip(items, upd):
                    full = DTensor.from_local(u, mesh, p.placements).full_tensor()
                    o = newton_schulz_ref(full, ns_steps) if not full.is_cuda else \
                        ops.batched_newton_schulz_orthogonalize(full.bfloat16()[None], ns_steps)[0]
                    shards.append(distribute_tensor(o, mesh, p.placements).to_local())
        else:
            pg = mesh.get_group()
            pad = (-len(items)) % world
            per = (len(items) + pad) // world
            lst = [u.bfloat16() for u in upd]
            lst += [torch.zeros(shard_rows, cols, device=lp[0].device, dtype=torch.bfloat16) for _ in range(pad)]
            send = torch.stack(lst).view(world, per, shard_rows, cols).contiguous()
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=pg)
            owned = recv.permute(1, 0, 2, 3).contiguous().view(per, rows, cols)
            orth = ops.batched_newton_schulz_orthogonalize(owned, ns_steps) if owned.is_cuda else \
                newton_schulz_ref(owned, ns_steps)
            back = orth.view(per, world, shard_rows, cols).permute(1, 0, 2, 3).contiguous()
            dist.all_to_all_single(recv, back, group=pg)
            shards = list(recv.view(per * world, shard_rows, cols)[: len(items)])
        if wd != 0.0:
            torch._foreach_mul_(lp, 1.0 - lr * wd)
        torch._foreach_add_(lp, [s.to(p.dtype) for s, p in zip(shards, lp)], alpha=-lr * lr_ratio((rows, cols), mode))


class AdamW(torch.optim.AdamW):
    """torch.optim.AdamW's state and group layout, stepped by one multi-tensor sm_100a
    kernel per group on CUDA (decoupled weight decay, bias correction)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, **kw):
        kw.pop("fused", None)
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, **kw)
        self.grad_scale: torch.Tensor | None = None  # as Muon.grad_scale

    @torch.no_grad()
    def step(self, closure=None):  # type: ignore[override]
        for group in self.param_groups:
            b1, b2 = group["betas"]
            by_dev: dict[tuple, list] = defaultdict(list)
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if len(st) == 0:
                    st["step"] = torch.zeros((), dtype=torch.float32)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["step"] += 1
                key = (p.device, p.grad.dtype, int(st["step"].item()) if not st["step"].is_cuda else -1)
                by_dev[key].append(p)
            for (dev, _, step), ps in by_dev.items():
                if step < 0:
                    step = int(self.state[ps[0]]["step"].item())
                local = [_local(p) for p in ps]
                grads = [_local(p.grad) for p in ps]
                ms = [_local(self.state[p]["exp_avg"]) for p in ps]
                vs = [_local(self.state[p]["exp_avg_sq"]) for p in ps]
                scale = self.grad_scale
                if local and local[0].is_cuda and all(t.dtype == torch.float32 for t in local):
                    ops.adamw_multi_tensor(local, [g.contiguous() for g in grads], ms, vs, step, group["lr"], b1, b2,
                                           group["eps"], group["weight_decay"], scale)
                else:
                    from ..ops.reference import adamw_ref

                    for p, g, m, v in zip(local, grads, ms, vs):
                        g = g.to(p.dtype) if scale is None else g.to(p.dtype) * scale
                        adamw_ref(p, g, m, v, step, group["lr"], b1, b2, group["eps"], group["weight_decay"])


def _local(t: torch.Tensor) -> torch.Tensor:
    return t.to_local() if _is_dtensor(t) else t


@dataclass
class ParameterGroups:
    muon: list[nn.Parameter]
    decay: list[nn.Parameter]
    no_decay: list[nn.Parameter]
    ngram: list[nn.Parameter]


def split_parameters(model: nn.Module, use_muon: bool) -> ParameterGroups:
    """Muon: 2-D weights inside blocks.  AdamW without decay: token embedding, output
    head and 1-D parameters.  n-gram tables: their own group.  AdamW with decay: the
    rest (e.g. 3-D convolution weights)."""
    groups = ParameterGroups([], [], [], [])
    seen: set[int] = set()
    for name, p in model.named_parameters():
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        if name.startswith("embed.ngram.tables."):
            groups.ngram.append(p)
            continue
        is_embedding = (name.startswith("embed.") and "proj" not in name) or name == "lm_head.weight"
        if is_embedding or p.ndim < 2:
            groups.no_decay.append(p)
        elif use_muon and p.ndim == 2:
            groups.muon.append(p)
        else:
            groups.decay.append(p)
    return groups


def build_optimizers(model: nn.Module, config: OptimizerConfig) -> list[torch.optim.Optimizer]:
    g = split_parameters(model, use_muon=config.name == "muon")
    out: list[torch.optim.Optimizer] = []
    if g.muon:
        out.append(Muon(g.muon, lr=config.muon_lr if config.muon_lr is not None else config.lr,
                        weight_decay=config.muon_weight_decay if config.muon_weight_decay is not None
                        else config.weight_decay,
                        momentum=config.muon_momentum, nesterov=config.muon_nesterov, ns_steps=config.muon_ns_steps,
                        adjust_lr=config.muon_adjust_lr))
    adam_groups = [
        {"params": g.decay, "weight_decay": config.weight_decay},
        {"params": g.no_decay, "weight_decay": 0.0},
        {"params": g.ngram, "weight_decay": config.ngram.weight_decay, "lr": config.lr * config.ngram.lr_scale},
    ]
    out.append(AdamW([x for x in adam_groups if x["params"]], lr=config.lr, betas=tuple(config.betas),
                     eps=config.eps))
    return out


def lr_multiplier(step: int, total_steps: int, config: ScheduleConfig) -> float:
    """Linear warmup, then cosine / WSD / constant (1-based step)."""
    warmup = min(total_steps, int(total_steps * config.warmup_ratio))
    if warmup and step <= warmup:
        return step / warmup

    def cosine(progress: float) -> float:
        progress = min(1.0, max(0.0, progress))
        return config.min_lr_ratio + (1 - config.min_lr_ratio) * 0.5 * (1 + math.cos(math.pi * progress))

    if config.kind == "constant":
        return 1.0
    if config.kind == "cosine":
        return cosine((step - warmup) / max(1, total_steps - warmup))
    decay = min(total_steps - warmup, int(total_steps * config.decay_ratio))
    start = total_steps - decay
    if decay == 0 or step <= start:
        return 1.0
    return cosine((step - start) / decay)


def set_lr(optimizers, base_lrs, multiplier: float) -> None:
    for opt, lrs in zip(optimizers, base_lrs):
        for group, base in zip(opt.param_groups, lrs):
            group["lr"] = base * multiplier
