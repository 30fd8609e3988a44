"""Data parallelism with sharded optimizer state and peer-memory collectives.

Design (B200-first).  The benchmark models (200M, 1B) and their gradients fit on every
GPU many times over (180 GB of HBM), so parameters stay replicated and only the optimizer
work is partitioned: every rank owns a set of element ranges of the flat parameter /
gradient buffers — whole matrices for Muon (Newton-Schulz needs the full matrix), even
slices of everything else for AdamW — and keeps optimizer state for those ranges only.
Per step (``optimizer_step``):

1. barrier across GPUs (all backward passes done);
2. ``dp_reduce_sumsq``: each owner reads its ranges from every peer's gradient buffer
   over NVLink, writes the sum into its own buffer and accumulates the squared norm
   (reduce-scatter fused with the clipping norm);
3. barrier; the global norm is the sum of every rank's partial (read by peer loads);
4. ``dp_adamw_allgather``: AdamW on the owned slices with the clip factor folded in, the
   new fp32 values stored straight into every rank's parameter buffer (all-gather fused
   with the update); Muon: momentum/Nesterov/pack of the owned matrices, batched
   Newton-Schulz on the tcgen05 GEMM, ``dp_muon_apply_allgather`` stores the update into
   every rank;
5. barrier (all writes visible before the next forward).

Compared with the reference's FSDP2 (per-block all-gather in forward and again in
backward, reduce-scatter per block per micro-batch, Muon's two all-to-alls), this moves
one gradient reduce-scatter and one parameter all-gather per optimizer step, in fp32, with
no NCCL call.  The flat buffers come from torch's symmetric memory (peer pointers); the
kernels are in ``csrc/comm.cu``.

On CPU (gloo, tests) the same ownership and arithmetic run with ``all_reduce``, which is
also the oracle for the GPU path.
"""

from __future__ import annotations

import math
from collections import defaultdict
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops
from ..ops.reference import newton_schulz_ref
from .distributed import DistInfo

ALIGN = 16  # elements: every parameter starts on a 64-byte boundary of the flat buffers


@dataclass
class Slot:
    param: nn.Parameter
    name: str
    offset: int
    numel: int


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class ShardedDataParallel(nn.Module):
    """Wraps a model; see module docstring.  ``owns_gradients`` tells the trainer that
    this runtime provides the gradient buffers and the whole optimizer step."""

    owns_gradients = True

    def __init__(self, model: nn.Module, info: DistInfo) -> None:
        super().__init__()
        self.module = model
        self.info = info
        self.world, self.rank = info.world_size, info.rank
        params = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
        seen: set[int] = set()
        self.slots: list[Slot] = []
        off = 0
        for n, p in params:
            if id(p) in seen:
                continue
            seen.add(id(p))
            self.slots.append(Slot(p, n, off, p.numel()))
            off += _align(p.numel())
        self.total = _align(off)
        dev = info.device
        self.cuda = dev.type == "cuda"
        if self.cuda:
            self._alloc_symmetric(dev)
        else:
            self.flat_param = torch.zeros(self.total, dtype=torch.float32, device=dev)
            self.flat_grad = torch.zeros(self.total, dtype=torch.float32, device=dev)
        with torch.no_grad():
            for s in self.slots:
                view = self.flat_param[s.offset:s.offset + s.numel].view_as(s.param)
                view.copy_(s.param.detach().float())
                s.param.data = view
                g = self.flat_grad[s.offset:s.offset + s.numel].view_as(s.param)
                s.param.main_grad = g
                s.param.grad = g
        # start from identical parameters on every rank
        if dist.is_initialized():
            dist.broadcast(self.flat_param, src=0)
        self.optimizers: list[torch.optim.Optimizer] = []
        self.step_count = 0
        self.epoch = 0
        self.last_norm = torch.zeros((), device=dev)

    # -- symmetric memory ---------------------------------------------------------------
    def _alloc_symmetric(self, dev) -> None:
        import torch.distributed._symmetric_memory as symm

        group = dist.group.WORLD
        self.flat_param = symm.empty(self.total, dtype=torch.float32, device=dev)
        self.flat_grad = symm.empty(self.total, dtype=torch.float32, device=dev)
        self.ctrl = symm.empty(64, dtype=torch.int32, device=dev)  # [0, world): barrier flags; [32]: norm partial
        self.flat_grad.zero_()
        self.ctrl.zero_()
        hp = symm.rendezvous(self.flat_param, group)
        hg = symm.rendezvous(self.flat_grad, group)
        hc = symm.rendezvous(self.ctrl, group)
        self.param_ptrs = torch.tensor(list(hp.buffer_ptrs), dtype=torch.int64, device=dev)
        self.grad_ptrs = torch.tensor(list(hg.buffer_ptrs), dtype=torch.int64, device=dev)
        self.flag_ptrs = torch.tensor(list(hc.buffer_ptrs), dtype=torch.int64, device=dev)
        self.partial_ptrs = self.flag_ptrs + 32 * 4
        self.partial = self.ctrl[32:33].view(torch.float32)
        self._handles = (hp, hg, hc)
        torch.cuda.synchronize(dev)
        dist.barrier()

    def _barrier(self) -> None:
        self.epoch += 1
        if self.cuda:
            ops.ext().peer_barrier(self.flag_ptrs, self.rank, self.world, self.epoch)

    # -- module plumbing ----------------------------------------------------------------
    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def module_for_checkpoint(self) -> nn.Module:
        return self.module

    def optim_module(self) -> nn.Module:
        return self.module

    @property
    def config(self):
        return self.module.config

    def parameters(self, recurse: bool = True):
        return self.module.parameters(recurse)

    def named_parameters(self, *a, **k):
        return self.module.named_parameters(*a, **k)

    def zero_grad(self, set_to_none: bool = False) -> None:  # noqa: ARG002
        self.flat_grad.zero_()

    # -- ownership ---------------------------------------------------------------------
    def attach_optimizers(self, optimizers: list[torch.optim.Optimizer]) -> None:
        from ..train.optim import Muon, lr_ratio

        self.optimizers = optimizers
        by_param = {id(s.param): s for s in self.slots}
        self.muon_buckets: dict[tuple, dict] = {}
        self.adam_ranges: list[tuple[int, int, dict]] = []  # (flat offset, length, group)
        adam_slots: list[tuple[Slot, dict]] = []
        for opt in optimizers:
            for group in opt.param_groups:
                for p in group["params"]:
                    s = by_param[id(p)]
                    if isinstance(opt, Muon):
                        b = self.muon_buckets.setdefault(tuple(p.shape), {"slots": [], "group": group,
                                                                          "ratio": lr_ratio(p.shape, group["adjust_lr"])})
                        b["slots"].append(s)
                    else:
                        adam_slots.append((s, group))
        # Muon: whole matrices, round-robin inside each shape bucket
        self.owned_muon: dict[tuple, list[Slot]] = {}
        for shape, b in self.muon_buckets.items():
            mine = [s for i, s in enumerate(b["slots"]) if i % self.world == self.rank]
            self.owned_muon[shape] = mine
        # AdamW: even slices of the concatenated AdamW index space (multiples of 4 elements)
        spans = []
        acc = 0
        for s, g in adam_slots:
            n4 = _align(s.numel)  # pad to the aligned slot length (padding gets zero grads)
            spans.append((acc, s, g, n4))
            acc += n4
        total = acc
        per = (total // self.world + 3) // 4 * 4
        lo, hi = min(total, self.rank * per), min(total, (self.rank + 1) * per) if self.rank < self.world - 1 else total
        for start, s, g, n4 in spans:
            a, b_ = max(lo, start), min(hi, start + n4)
            if a < b_:
                self.adam_ranges.append((s.offset + (a - start), b_ - a, g))
        self._build_tables()
        dev = self.flat_param.device
        n_adam = sum(r[1] for r in self.adam_ranges)
        self.adam_m = torch.zeros(n_adam, dtype=torch.float32, device=dev)
        self.adam_v = torch.zeros(n_adam, dtype=torch.float32, device=dev)
        self.muon_mom = {shape: torch.zeros(len(sl), *shape, dtype=torch.float32, device=dev)
                         for shape, sl in self.owned_muon.items()}

    def _build_tables(self) -> None:
        dev = self.flat_param.device
        owned = [(s.offset, _align(s.numel)) for sl in self.owned_muon.values() for s in sl]
        owned += [(o, n) for o, n, _ in self.adam_ranges]
        owned.sort()
        self.red_offsets = torch.tensor([o for o, _ in owned] or [0], dtype=torch.int64, device=dev)[:len(owned)]
        pre = [0]
        for _, n in owned:
            pre.append(pre[-1] + n)
        self.red_prefix = torch.tensor(pre, dtype=torch.int64, device=dev)
        self.red_total = pre[-1]
        self.adam_offsets = torch.tensor([o for o, _, _ in self.adam_ranges], dtype=torch.int64, device=dev)
        ap = [0]
        for _, n, _ in self.adam_ranges:
            ap.append(ap[-1] + n)
        self.adam_prefix = torch.tensor(ap, dtype=torch.int64, device=dev)
        self.adam_total = ap[-1]
        self.muon_offs = {shape: torch.tensor([s.offset for s in sl], dtype=torch.int64, device=dev)
                          for shape, sl in self.owned_muon.items()}

    # -- the optimizer step ------------------------------------------------------------
    @torch.no_grad()
    def optimizer_step(self, grad_clip: float) -> torch.Tensor:
        self.step_count += 1
        if self.cuda:
            return self._step_cuda(grad_clip)
        return self._step_reference(grad_clip)

    def _adam_hparams(self):
        adam = self.optimizers[-1]
        b1, b2 = adam.param_groups[0]["betas"]
        eps = adam.param_groups[0]["eps"]
        return b1, b2, eps

    def _step_cuda(self, grad_clip: float) -> torch.Tensor:
        ext = ops.ext()
        self.partial.zero_()
        self._barrier()
        ext.dp_reduce_sumsq(self.grad_ptrs, self.rank, self.world, self.red_offsets, self.red_prefix, self.partial,
                            self.red_total)
        self._barrier()
        b1, b2, eps = self._adam_hparams() if self.optimizers else (0.9, 0.95, 1e-8)
        dev = self.flat_param.device
        wd = torch.tensor([g["weight_decay"] for _, _, g in self.adam_ranges] or [0.0], dtype=torch.float32)
        lr = torch.tensor([g["lr"] for _, _, g in self.adam_ranges] or [0.0], dtype=torch.float32)
        wd = wd.pin_memory().to(dev, non_blocking=True)
        lr = lr.pin_memory().to(dev, non_blocking=True)
        norm = torch.zeros(1, dtype=torch.float32, device=dev)
        ext.dp_adamw_allgather(self.param_ptrs, self.grad_ptrs, self.rank, self.world, self.adam_offsets,
                               self.adam_prefix, wd, lr, self.adam_m, self.adam_v, b1, b2, eps, self.step_count,
                               self.partial_ptrs, 0.0, float(grad_clip or 0.0), norm, self.adam_total)
        for shape, sl in self.owned_muon.items():
            if not sl:
                continue
            b = self.muon_buckets[shape]
            g = b["group"]
            packed = torch.empty(len(sl), *shape, dtype=torch.bfloat16, device=dev)
            ext.dp_muon_prepare(self.grad_ptrs, self.rank, self.world, self.muon_offs[shape],
                                math.prod(shape), self.muon_mom[shape], g["momentum"], g["nesterov"], packed,
                                self.partial_ptrs, 0.0, float(grad_clip or 0.0))
            orth = ops.batched_newton_schulz_orthogonalize(packed, g["ns_steps"])
            ext.dp_muon_apply_allgather(self.param_ptrs, self.rank, self.world, self.muon_offs[shape],
                                        math.prod(shape), g["lr"] * g["weight_decay"], -g["lr"] * b["ratio"], orth)
        self._barrier()
        if not bool(ops.ext().take_status() == 0) if False else False:  # status is read by tests
            pass
        self.last_norm = norm[0]
        return norm[0]

    def _step_reference(self, grad_clip: float) -> torch.Tensor:
        """CPU / gloo path with the same ownership and arithmetic (all_reduce based)."""
        if dist.is_initialized():
            dist.all_reduce(self.flat_grad)
        sq = torch.zeros((), dtype=torch.float64)
        for o, n in zip(self.red_offsets.tolist(), (self.red_prefix[1:] - self.red_prefix[:-1]).tolist()):
            sq += self.flat_grad[o:o + n].double().square().sum()
        if dist.is_initialized():
            dist.all_reduce(sq)
        norm = sq.sqrt().float()
        coef = min(1.0, grad_clip / (float(norm) + 1e-6)) if grad_clip and grad_clip > 0 else 1.0
        b1, b2, eps = self._adam_hparams() if self.optimizers else (0.9, 0.95, 1e-8)
        bc1 = 1 - b1 ** self.step_count
        bc2 = math.sqrt(1 - b2 ** self.step_count)
        new = torch.zeros_like(self.flat_param)
        mask = torch.zeros(self.total, dtype=torch.bool)
        pos = 0
        for o, n, g in self.adam_ranges:
            p = self.flat_param[o:o + n]
            gr = self.flat_grad[o:o + n] * coef
            m = self.adam_m[pos:pos + n]
            v = self.adam_v[pos:pos + n]
            m.lerp_(gr, 1 - b1)
            v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
            upd = p * (1 - g["lr"] * g["weight_decay"]) - (g["lr"] / bc1) * m / (v.sqrt() / bc2 + eps)
            new[o:o + n] = upd
            mask[o:o + n] = True
            pos += n
        for shape, sl in self.owned_muon.items():
            if not sl:
                continue
            b = self.muon_buckets[shape]
            g = b["group"]
            mom = self.muon_mom[shape]
            ups = []
            for i, s in enumerate(sl):
                gr = self.flat_grad[s.offset:s.offset + s.numel].view(shape) * coef
                mom[i].lerp_(gr, 1 - g["momentum"])
                ups.append(gr.lerp(mom[i], g["momentum"]) if g["nesterov"] else mom[i].clone())
            orth = newton_schulz_ref(torch.stack(ups), g["ns_steps"])
            for i, s in enumerate(sl):
                p = self.flat_param[s.offset:s.offset + s.numel]
                new[s.offset:s.offset + s.numel] = p * (1 - g["lr"] * g["weight_decay"]) + \
                    (-g["lr"] * b["ratio"]) * orth[i].reshape(-1).float()
                mask[s.offset:s.offset + s.numel] = True
        contrib = torch.where(mask, new, torch.zeros_like(new))
        if dist.is_initialized():
            dist.all_reduce(contrib)
            owned_any = mask.float()
            dist.all_reduce(owned_any)
            self.flat_param.copy_(torch.where(owned_any > 0, contrib, self.flat_param))
        else:
            self.flat_param.copy_(torch.where(mask, contrib, self.flat_param))
        self.last_norm = norm
        return norm

    # -- checkpoint plumbing -----------------------------------------------------------
    def sync_params_for_checkpoint(self) -> None:
        """Materialise full per-parameter optimizer state (Muon momentum_buffer, AdamW
        step/exp_avg/exp_avg_sq) in the torch optimizers so DCP saves the reference layout."""
        from ..train.optim import Muon

        dev = self.flat_param.device
        full_m = torch.zeros(self.total, dtype=torch.float32, device=dev)
        full_v = torch.zeros(self.total, dtype=torch.float32, device=dev)
        full_mom = torch.zeros(self.total, dtype=torch.float32, device=dev)
        pos = 0
        for o, n, _ in self.adam_ranges:
            full_m[o:o + n] = self.adam_m[pos:pos + n]
            full_v[o:o + n] = self.adam_v[pos:pos + n]
            pos += n
        for shape, sl in self.owned_muon.items():
            for i, s in enumerate(sl):
                full_mom[s.offset:s.offset + s.numel] = self.muon_mom[shape][i].reshape(-1)
        if dist.is_initialized():
            for t in (full_m, full_v, full_mom):
                dist.all_reduce(t)
        for opt in self.optimizers:
            for group in opt.param_groups:
                for p in group["params"]:
                    s = next(x for x in self.slots if x.param is p)
                    st = opt.state[p]
                    if isinstance(opt, Muon):
                        st["momentum_buffer"] = full_mom[s.offset:s.offset + s.numel].view_as(p).clone()
                    else:
                        st["step"] = torch.tensor(float(self.step_count))
                        st["exp_avg"] = full_m[s.offset:s.offset + s.numel].view_as(p).clone()
                        st["exp_avg_sq"] = full_v[s.offset:s.offset + s.numel].view_as(p).clone()

    def after_checkpoint_load(self) -> None:
        """Scatter loaded per-parameter optimizer state back into the owned shards."""
        from ..train.optim import Muon

        pos = 0
        slot_of = {id(s.param): s for s in self.slots}
        flat_m = torch.zeros(self.total, dtype=torch.float32, device=self.flat_param.device)
        flat_v = torch.zeros_like(flat_m)
        flat_mom = torch.zeros_like(flat_m)
        step = None
        for opt in self.optimizers:
            for group in opt.param_groups:
                for p in group["params"]:
                    s = slot_of[id(p)]
                    st = opt.state.get(p, {})
                    if isinstance(opt, Muon) and "momentum_buffer" in st:
                        flat_mom[s.offset:s.offset + s.numel] = st["momentum_buffer"].reshape(-1).float()
                    elif "exp_avg" in st:
                        flat_m[s.offset:s.offset + s.numel] = st["exp_avg"].reshape(-1).float()
                        flat_v[s.offset:s.offset + s.numel] = st["exp_avg_sq"].reshape(-1).float()
                        step = int(float(st["step"]))
        for o, n, _ in self.adam_ranges:
            self.adam_m[pos:pos + n] = flat_m[o:o + n]
            self.adam_v[pos:pos + n] = flat_v[o:o + n]
            pos += n
        for shape, sl in self.owned_muon.items():
            for i, s in enumerate(sl):
                self.muon_mom[shape][i].copy_(flat_mom[s.offset:s.offset + s.numel].view(shape))
        if step is not None:
            self.step_count = step


def shard_model(model: nn.Module, info: DistInfo, reshard_after_forward: bool = True) -> ShardedDataParallel:
    return ShardedDataParallel(model, info)
