"""Sharded data parallelism over NVLink peer memory: parameter-sharded (default) or
optimizer-sharded.

Layout.  Parameters are split into two kinds at ``attach_optimizers`` time:

* **Row-sharded weights** (``shard_params=True``, every Muon-optimised ``nn.Linear``
  weight whose shape allows it): like FSDP2's dim-0 sharding, rank ``r`` keeps rows
  ``[r*R, (r+1)*R)`` of the fp32 master (``R = ceil(rows / world)``) plus a bf16 copy of
  them; no rank holds the full weight between uses.  A forward linear runs
  ``gemm_gather`` (``csrc/gemm.cu``): extra warps of the tcgen05 GEMM copy the shards from
  the owners' memory into a local bf16 buffer while the tensor cores start on the rows
  this rank owns, and the TMA producer waits per 64-row chunk.  The data-gradient GEMM of
  the backward pass reuses that buffer if it still holds the weight, else gathers again
  inside the GEMM (the reduction loop starts at the local rows).  ``reshard_after_forward``
  decides the buffers: a ring of two per weight shape (each use gathers, the FSDP2
  default) or one per weight (one gather per optimizer step).
* **Replicated parameters** (embeddings, the output head, norms, gates, AdamW weights and
  Muon weights that cannot be row-sharded): one fp32 copy per rank, optimizer state
  sharded.

Gradients accumulate in one flat fp32 buffer per rank (full size; the GEMM epilogues add
into it).  Each optimizer step (``optimizer_step``):

1. peer barrier (every rank finished its backward passes);
2. ``dp_reduce_sumsq``: each rank sums, from every peer's gradient buffer, the element
   ranges it owns (whole matrices for Muon, even slices of the AdamW space) and
   accumulates their squared norm: the reduce-scatter fused with the clipping norm.  With
   NVSwitch multicast (NVLS) available, ``dp_reduce_sumsq_multimem`` reads each owned
   element once through the switch, which adds up every rank's copy (``multimem.ld_reduce``);
3. peer barrier; the clip coefficient is formed on the device from all partial norms;
4. ``dp_adamw_allgather``: AdamW on the owned slices, the result stored into every rank's
   replicated copy.  Muon: momentum / Nesterov / bf16 pack of the owned matrices, batched
   Newton-Schulz on the tcgen05 GEMM, then ``dp_muon_apply_shards`` writes each row of the
   update into its owner's fp32 master and bf16 shard (row-sharded weights) or
   ``dp_muon_apply_allgather`` into every rank's copy (replicated);
5. peer barrier (all writes visible before the next forward's gathers).

No NCCL call is on this path: the buffers are torch symmetric memory (peer pointers) and
every transfer is a 16-byte peer load or store inside these kernels.  The reference
shards every block with FSDP2 (``src/myk_llm/train/distributed.py:108-134``) and moves
the same data with NCCL all-gathers and reduce-scatters.

On CPU (gloo, tests) the same layout, ownership and arithmetic run with collectives,
which is also the oracle for the GPU path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops
from ..ops.linear import SKINNY_MAX_ROWS
from ..ops.reference import newton_schulz_ref
from .distributed import DistInfo

ALIGN = 16  # elements: every slot starts on a 64-byte (fp32) / 32-byte (bf16) boundary


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class Slot:
    param: nn.Parameter
    name: str
    goff: int            # offset of the full-size gradient in the flat gradient buffer
    poff: int            # offset in the flat fp32 parameter buffer (full copy or this rank's rows)
    numel: int           # full element count
    sharded: bool = False
    rows: int = 0
    cols: int = 0
    rows_per_rank: int = 0
    boff: int = 0        # offset of the bf16 shard in the flat bf16 buffer
    weight: "ShardedWeight | None" = field(default=None, repr=False)
    mx: bool = False     # MXFP8 linear: its rows' fp8 copies are what the ranks gather
    moff: int = 0        # offset of those copies in the flat fp8 buffer (bytes)

    @property
    def shard_numel(self) -> int:
        return self.rows_per_rank * self.cols


class GatherBuffer:
    """A local bf16 buffer a row-sharded weight is gathered into, with the per-64-row
    arrival counters of the fused gather (zeroed once; each gather raises them by a fixed
    amount, so they never need resetting) and the identity of what it holds."""

    def __init__(self, rows: int, cols: int, device: torch.device) -> None:
        self.w = torch.empty(rows, cols, dtype=torch.bfloat16, device=device)
        self.ready = torch.zeros(max(1, (rows + 63) // 64), dtype=torch.int32, device=device)
        self.epoch = 0
        self.holder: tuple[int, int] | None = None


class UseTrace:
    """Order in which row-sharded weights are used by forward products, recorded over one
    optimizer step and replayed as prefetch hints in the next (a wrong hint only costs a
    gather: every use checks what its buffer holds)."""

    def __init__(self) -> None:
        self.previous: list["ShardedWeight"] = []
        self.current: list["ShardedWeight"] = []

    def next_after(self, w: "ShardedWeight") -> "ShardedWeight | None":
        pos = len(self.current)
        self.current.append(w)
        if pos + 1 < len(self.previous) and self.previous[pos] is w:
            return self.previous[pos + 1]
        return None

    def end_step(self) -> None:
        self.previous, self.current = self.current, []


class ShardedWeight:
    """Run-time handle of one row-sharded weight, attached to its parameter as
    ``_mykb_shard``; ``ops.linear`` routes the parameter's products through it."""

    def __init__(self, rt: "ShardedDataParallel", slot: Slot, buf: GatherBuffer | None) -> None:
        self.rt = rt
        self.slot = slot
        self.buf = buf
        self.rows, self.cols = slot.rows, slot.cols
        self._cpu_full: tuple[int, torch.Tensor] | None = None
        self._mx: list[torch.Tensor] | None = None
        self._mx_version = -1

    def mx_operands(self) -> list[torch.Tensor]:
        """[W q0, s0, W^T q1, s1] (E4M3) of an MXFP8 weight, gathered once per optimizer step
        from every rank's fp8 copies of its rows (``mx_shard_gather``: 16-byte peer loads of
        fp8 values and E8M0 scale atoms, about half the bytes of a bf16 gather)."""
        rt, s = self.rt, self.slot
        if self._mx is None:
            dev = rt.info.device
            n, k = s.rows, s.cols
            u8 = dict(dtype=torch.uint8, device=dev)
            self._mx = [torch.empty(n, k, **u8), torch.empty(n * k // 32, **u8), torch.empty(k, n, **u8),
                        torch.empty(n * k // 32, **u8)]
            self._mx_bases = rt.mx_bases + s.moff
        if self._mx_version != rt.version:
            ops.ext().mx_shard_gather(self._mx_bases, s.rows_per_rank, s.cols, s.rows, *self._mx)
            self._mx_version = rt.version
        return self._mx

    # -- CUDA --------------------------------------------------------------------------
    def _key(self) -> tuple[int, int]:
        return (id(self), self.rt.version)

    def holds(self) -> bool:
        return self.buf.holder == self._key()

    def _gather_args(self):
        """Arguments of a gather into this weight's buffer; marks the buffer as holding it
        (every later use is ordered after the gather on the stream)."""
        rt, s = self.rt, self.slot
        self.buf.epoch += 1
        self.buf.holder = self._key()
        return self.buf.w, rt.bf16_ptrs, s.boff, s.rows_per_rank, rt.rank, self.buf.ready, self.buf.epoch

    def can_prefetch_during(self, other: "ShardedWeight") -> bool:
        return self is not other and not self.holds() and self.buf is not other.buf

    def forward_gemm(self, x2: torch.Tensor) -> torch.Tensor:
        """y = x W^T.  W not gathered yet: the GEMM gathers it and waits per 64 rows.  W
        gathered: the GEMM's gather warps prefetch the weight the next forward product
        uses (learned from the previous step's order of uses)."""
        rt = self.rt
        nxt = rt.trace.next_after(self)
        y = torch.empty(x2.shape[0], self.rows, dtype=torch.bfloat16, device=x2.device)
        if not self.holds():
            ops.ext().gemm_gather(x2, self.buf.w, y, False, False, False, *self._gather_args())
        elif nxt is not None and nxt.can_prefetch_during(self):
            ops.ext().gemm_gather(x2, self.buf.w, y, False, False, False, *nxt._gather_args())
        else:
            ops.gemm(x2, self.buf.w, out=y)
        return y

    def backward_gemms(self, dy2: torch.Tensor, x2: torch.Tensor, main_grad: torch.Tensor | None,
                       need_dx: bool) -> torch.Tensor | None:
        """Weight gradient (accumulated into ``main_grad``) and data gradient ``dy W``.  If W
        was released since the forward, the weight-gradient GEMM, which does not need W,
        gathers it with its spare warps, so the data-gradient GEMM finds it local."""
        ext = ops.ext()
        if main_grad is not None:
            if not self.holds() and need_dx:
                ext.gemm_gather(dy2, x2, main_grad, True, True, True, *self._gather_args())
            else:
                ops.gemm(dy2, x2, a_major="mn", b_major="mn", out=main_grad, accumulate=True)
        if not need_dx:
            return None
        dx = torch.empty(dy2.shape[0], self.cols, dtype=torch.bfloat16, device=dy2.device)
        if self.holds():
            ops.gemm(dy2, self.buf.w, b_major="mn", out=dx)
        else:
            ext.gemm_gather(dy2, self.buf.w, dx, False, True, False, *self._gather_args())
        return dx

    def full(self) -> torch.Tensor:
        """The whole bf16 weight (gathered by the standalone kernel if needed)."""
        if not self.holds():
            ops.ext().shard_gather(*self._gather_args())
        return self.buf.w

    # -- CPU (gloo) --------------------------------------------------------------------
    def linear(self, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        """y = x W^T through this handle (``ops.linear`` calls it for sharded parameters)."""
        if not x.is_cuda:
            return _ShardedLinearCPU.apply(x, weight, self)
        if self.slot.mx and x.numel() // x.shape[-1] > SKINNY_MAX_ROWS:
            from ..ops.mxfp8 import mx_linear  # fp8-gathered operands (``mx_operands``)

            return mx_linear(x, weight, weight._mykb_mxfp8)
        return _ShardedLinear.apply(x, weight, self)

    def full_cpu(self) -> torch.Tensor:
        """fp32 full weight on CPU, all-gathered from the ranks' master rows."""
        if self._cpu_full is not None and self._cpu_full[0] == self.rt.version:
            return self._cpu_full[1]
        full = self.rt.gather_full_fp32(self.slot)
        self._cpu_full = (self.rt.version, full)
        return full


class _ShardedLinear(torch.autograd.Function):
    """y = x W^T for a row-sharded W: fused gather GEMMs forward and for the data gradient,
    weight gradient accumulated in fp32 into the full-size gradient slot."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, shard: ShardedWeight):
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        if x2.shape[0] <= SKINNY_MAX_ROWS:
            wb = shard.full()
            y = torch.empty(x2.shape[0], shard.rows, dtype=torch.bfloat16, device=x2.device)
            ops.ext().gemm_skinny(x2, wb, y)
        else:
            y = shard.forward_gemm(x2)
        ctx.save_for_backward(x2)
        ctx.shard, ctx.w = shard, w
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        return y.view(*x.shape[:-1], shard.rows)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        (x2,) = ctx.saved_tensors
        shard, w = ctx.shard, ctx.w
        dy2 = dy.reshape(-1, shard.rows)
        if dy2.dtype != torch.bfloat16:
            dy2 = dy2.to(torch.bfloat16)
        dy2 = dy2.contiguous()
        main = w.main_grad if ctx.needs_input_grad[1] else None
        dx = shard.backward_gemms(dy2, x2, main, ctx.needs_input_grad[0])
        if dx is not None:
            dx = dx.view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        return dx, None, None


class _ShardedLinearCPU(torch.autograd.Function):
    """CPU statement of the same product: the full weight is all-gathered from the ranks'
    fp32 master rows, the weight gradient is added into the full-size gradient slot."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, shard: ShardedWeight):
        full = shard.full_cpu().to(x.dtype)
        ctx.save_for_backward(x)
        ctx.shard, ctx.w = shard, w
        return torch.nn.functional.linear(x, full)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        (x,) = ctx.saved_tensors
        full = ctx.shard.full_cpu().to(dy.dtype)
        dx = dy @ full if ctx.needs_input_grad[0] else None
        if ctx.needs_input_grad[1]:
            k = x.shape[-1]
            ctx.w.main_grad.add_((dy.reshape(-1, dy.shape[-1]).float().t() @ x.reshape(-1, k).float()))
        return dx, None, None


class TableShards:
    """Row-sharded hashed n-gram tables (GPU, two or more ranks).

    Rank ``r`` owns rows ``[r*R, (r+1)*R)`` (``R = ceil(buckets / world)``) of every order's
    table: the fp32 master and the gradient rows live in symmetric memory (peers read the
    master rows and add into the gradient rows), the AdamW moments are local.  The
    embedding forward (``ngram_embed_fwd_shard``) hashes each position and reads its rows
    from their owners; the backward (``ngram_embed_bwd_shard``) adds the position's
    gradient into the owners' rows.  At the optimizer step each rank adds its gradient
    shard's squared norm to the global clipping norm and runs AdamW on its rows, zeroing
    the gradient rows for the next step (here, between the step's barriers: a peer may add
    into them as soon as the step is over).  Only the rows a step's tokens touch cross
    NVLink, where a replicated table would reduce and gather the whole table.  The tables
    keep their parameters' full shapes and optimizer-state keys in checkpoints.
    """

    def __init__(self, rt: "ShardedDataParallel", params: list[nn.Parameter], orders: list[int]) -> None:
        self.rt = rt
        self.params = params
        self.orders = list(orders)
        self.buckets, self.dim = params[0].shape
        if any(tuple(p.shape) != (self.buckets, self.dim) for p in params) or self.dim % 4:
            raise ValueError("row-sharded n-gram tables need one shape and a width that is a multiple of 4")
        world, rank = rt.world, rt.rank
        self.rows_per_rank = -(-self.buckets // world)
        self.stride = _align(self.rows_per_rank * self.dim)  # elements between orders in a rank's buffer
        total = self.stride * len(params)
        dev = rt.info.device
        if rt.cuda:
            import torch.distributed._symmetric_memory as symm

            self.param = symm.empty(total, dtype=torch.float32, device=dev)
            self.grad = symm.empty(total, dtype=torch.float32, device=dev)
            self.param.zero_()
            self.grad.zero_()
            self._handles = [symm.rendezvous(t, dist.group.WORLD) for t in (self.param, self.grad)]
            # base addresses stay on the host: the launch reads them without a device sync
            self.param_bases = torch.tensor(list(self._handles[0].buffer_ptrs), dtype=torch.int64)
            self.grad_bases = torch.tensor(list(self._handles[1].buffer_ptrs), dtype=torch.int64)
        else:  # gloo: the same ownership with collectives instead of peer memory
            self.param = torch.zeros(total, dtype=torch.float32, device=dev)
            self.grad = torch.zeros(total, dtype=torch.float32, device=dev)
        self.m = torch.zeros(total, dtype=torch.float32, device=dev)
        self.v = torch.zeros(total, dtype=torch.float32, device=dev)
        self.lo = rank * self.rows_per_rank
        self.hi = min(self.buckets, self.lo + self.rows_per_rank)
        with torch.no_grad():
            for j, p in enumerate(params):
                full = p.detach().float().contiguous()
                dist.broadcast(full, src=0)
                if self.hi > self.lo:
                    self.shard(self.param, j)[:self.hi - self.lo].copy_(full[self.lo:self.hi])
                p.data = torch.zeros(1, dtype=torch.float32, device=dev).expand(self.buckets, self.dim)
                p._mykb_table = self
                p.main_grad = None
                p.grad = None
        self.group: dict | None = None

    def shard(self, buf: torch.Tensor, j: int) -> torch.Tensor:
        return buf[j * self.stride:j * self.stride + self.rows_per_rank * self.dim].view(self.rows_per_rank, self.dim)

    # -- embedding kernels -----------------------------------------------------------------
    def forward(self, tokens: torch.Tensor, context: int):
        return ops.ext().ngram_embed_fwd_shard(tokens, self.param_bases, self.stride * 4, self.rows_per_rank,
                                               self.buckets, self.dim, self.orders, context)

    def backward(self, rows: torch.Tensor, dout: torch.Tensor) -> None:
        ops.ext().ngram_embed_bwd_shard(rows, dout, self.grad_bases, self.stride * 4, self.rows_per_rank,
                                        self.buckets)

    # -- CPU (gloo) path -----------------------------------------------------------------
    def lookup_cpu(self, ids: torch.Tensor) -> torch.Tensor:
        """Sum over the orders of the rows ``ids`` (orders, ...) addresses in the stacked
        tables; forward from the all-gathered tables, backward adds the rank-summed gradient
        of this rank's rows into its shard."""
        return _TableLookupCPU.apply(ids, self, *self.params)  # the parameters make autograd call backward

    # -- optimizer step (between the runtime's barriers) -------------------------------------
    def add_sumsq(self, partial: torch.Tensor) -> None:
        ops.ext().shard_sumsq(self.grad, partial)

    def adamw(self, step: int, b1: float, b2: float, eps: float, clip: float) -> None:
        g = self.group or {"lr": 0.0, "weight_decay": 0.0}
        ops.ext().shard_adamw(self.param, self.grad, self.m, self.v, g["lr"], g["weight_decay"], b1, b2, eps, step,
                              self.rt.partial_ptrs, self.rt.world, clip)

    # -- checkpoints ---------------------------------------------------------------------
    def gather(self, buf: torch.Tensor, j: int) -> torch.Tensor:
        mine = self.shard(buf, j).contiguous()
        parts = [torch.empty_like(mine) for _ in range(self.rt.world)]
        dist.all_gather(parts, mine)
        return torch.cat(parts, 0)[:self.buckets]

    def scatter(self, buf: torch.Tensor, j: int, full: torch.Tensor) -> None:
        dst = self.shard(buf, j)
        dst.zero_()
        if self.hi > self.lo:
            dst[:self.hi - self.lo].copy_(full[self.lo:self.hi].to(dst.dtype))

    def materialise(self) -> None:
        with torch.no_grad():
            for j, p in enumerate(self.params):
                p.data = self.gather(self.param, j).contiguous()

    def dematerialise(self) -> None:
        dev = self.rt.info.device
        for p in self.params:
            p.data = torch.zeros(1, dtype=torch.float32, device=dev).expand(self.buckets, self.dim)

    def memory_bytes(self) -> int:
        return 4 * (self.param.numel() + self.grad.numel() + self.m.numel() + self.v.numel())

    def step_cpu(self, step: int, b1: float, b2: float, eps: float, coef: float) -> None:
        """AdamW on this rank's rows (the same rule as ``shard_adamw``), gradient rows zeroed."""
        g = self.group or {"lr": 0.0, "weight_decay": 0.0}
        lr, wd = g["lr"], g["weight_decay"]
        gr = self.grad * coef
        self.m.lerp_(gr, 1 - b1)
        self.v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
        bc1, bc2 = 1 - b1 ** step, math.sqrt(1 - b2 ** step)
        self.param.mul_(1 - lr * wd).sub_((lr / bc1) * self.m / (self.v.sqrt() / bc2 + eps))
        self.grad.zero_()


class _TableLookupCPU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids: torch.Tensor, shards: "TableShards", *params):
        ctx.shards = shards
        ctx.save_for_backward(ids)
        out = None
        for j in range(len(shards.params)):
            full = shards.gather(shards.param, j)
            rows = full[ids[j] - j * shards.buckets]
            out = rows if out is None else out + rows
        return out

    @staticmethod
    def backward(ctx, dout: torch.Tensor):
        (ids,) = ctx.saved_tensors
        t = ctx.shards
        d = dout.reshape(-1, dout.shape[-1]).float()
        for j in range(len(t.params)):
            dense = torch.zeros(t.buckets, t.dim, dtype=torch.float32)
            dense.index_add_(0, (ids[j] - j * t.buckets).reshape(-1), d)
            dist.all_reduce(dense)
            if t.hi > t.lo:
                t.shard(t.grad, j)[:t.hi - t.lo].add_(dense[t.lo:t.hi])
        return (None, None, *(None for _ in t.params))


class ShardedDataParallel(nn.Module):
    """Wraps a model; see module docstring.  ``owns_gradients`` tells the trainer that this
    runtime provides the gradient buffers and the whole optimizer step."""

    owns_gradients = True

    def __init__(self, model: nn.Module, info: DistInfo, shard_params: bool = True,
                 reshard_after_forward: bool = True) -> None:
        super().__init__()
        self.module = model
        self.info = info
        self.world, self.rank = info.world_size, info.rank
        self.shard_params = shard_params
        self.reshard_after_forward = reshard_after_forward
        self.cuda = info.device.type == "cuda"
        self.optimizers: list[torch.optim.Optimizer] = []
        self.step_count = 0
        self.epoch = 0
        self.version = 0  # bumped by every optimizer step: gathered copies are stale after it
        self.last_norm = torch.zeros((), device=info.device)
        self.slots: list[Slot] = []
        self._linear_weights = {id(m.weight) for m in model.modules() if type(m) is nn.Linear}
        self.trace = UseTrace()
        self.grad_mc = 0  # NVSwitch multicast address of the gradient buffer (0: peer loads)
        self.tables: TableShards | None = None  # row-sharded n-gram tables
        self.table_ids: set[int] = set()

    # -- module plumbing ----------------------------------------------------------------
    def forward(self, *args, **kwargs):
        if not self.slots:
            raise RuntimeError("ShardedDataParallel: attach_optimizers() must run before the first forward")
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

    # -- layout -------------------------------------------------------------------------
    def _shardable(self, p: nn.Parameter) -> bool:
        if not self.shard_params or self.world < 2 or p.dim() != 2 or id(p) not in self._linear_weights:
            return False
        rows, cols = p.shape
        if getattr(p, "_mykb_mxfp8", None) is not None:
            # MXFP8 linears: row shards of 128-row multiples, gathered as fp8 + E8M0 scales
            return self.cuda and rows % 128 == 0 and cols % 128 == 0
        if getattr(p, "_mykb_fp8", None) is not None:
            return False  # per-tensor / per-row float8 linears quantise their own replicated master
        return rows % 8 == 0 and cols % 8 == 0 and rows >= self.world

    def attach_optimizers(self, optimizers: list[torch.optim.Optimizer]) -> None:
        from ..train.optim import Muon, lr_ratio

        self.optimizers = optimizers
        muon_ids = {id(p) for o in optimizers if isinstance(o, Muon) for g in o.param_groups for p in g["params"]}
        names = {id(p): n for n, p in self.module.named_parameters()}
        ordered: list[nn.Parameter] = []
        seen: set[int] = set()
        for o in optimizers:
            for g in o.param_groups:
                for p in g["params"]:
                    if id(p) not in seen:
                        seen.add(id(p))
                        ordered.append(p)
        for _, p in self.module.named_parameters():  # trainable parameters no optimizer holds
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                ordered.append(p)
        table_params, table_orders = self._ngram_tables(muon_ids)
        self.table_ids = {id(p) for p in table_params}
        rep = [p for p in ordered if id(p) not in self.table_ids and not (id(p) in muon_ids and self._shardable(p))]
        shd = [p for p in ordered if id(p) in muon_ids and self._shardable(p)]
        # replicated slots: the same offset in the gradient and parameter buffers
        off = 0
        for p in rep:
            self.slots.append(Slot(p, names.get(id(p), "?"), off, off, p.numel()))
            off += _align(p.numel())
        self.rep_total = off
        goff, poff, boff, moff = off, off, 0, 0
        for p in shd:
            rows, cols = p.shape
            r = -(-rows // self.world)
            mx = getattr(p, "_mykb_mxfp8", None) is not None
            if mx:
                r = -(-r // 128) * 128
            s = Slot(p, names.get(id(p), "?"), goff, poff, p.numel(), True, rows, cols, r, boff, mx=mx, moff=moff)
            self.slots.append(s)
            goff += _align(p.numel())
            poff += _align(r * cols)
            boff += _align(r * cols)
            if mx:
                moff += -(-(2 * r * cols + r * cols // 16) // 512) * 512
        self.grad_total, self.param_total, self.bf16_total = _align(goff), _align(poff), _align(max(boff, ALIGN))
        self.mx_total = moff
        self._allocate()
        self._load_params_into_buffers()
        self.tables = TableShards(self, table_params, table_orders) if table_params else None
        self._build_ownership(optimizers, Muon, lr_ratio)
        self._quantize_mx_shards(sync=True)

    def _quantize_mx_shards(self, sync: bool = False) -> None:
        """MXFP8 copies (both blockings, E4M3) of this rank's rows of every MXFP8 weight, into
        symmetric memory where the other ranks' gathers read them; then a barrier."""
        mx = [s for s in self.slots if s.mx]
        if not mx or not self.cuda:
            return
        ext = ops.ext()
        for s in mx:
            r, k = s.rows_per_rank, s.cols
            rk = r * k
            base = self.flat_mx[s.moff:s.moff + 2 * rk + rk // 16]
            ext.mx_quantize_into(self.flat_bf16[s.boff:s.boff + rk].view(r, k), False, base[:rk],
                                 base[rk:rk + rk // 32], base[rk + rk // 32:2 * rk + rk // 32],
                                 base[2 * rk + rk // 32:])
        if sync:
            torch.cuda.synchronize(self.info.device)
            dist.barrier()
        else:
            self._barrier()

    def _ngram_tables(self, muon_ids: set[int]) -> tuple[list[nn.Parameter], list[int]]:
        """The hashed n-gram tables to row-shard: GPU, two or more ranks, parameter sharding
        on, dense (not lazily updated) tables trained by AdamW."""
        from ..models.embeddings import NgramEmbedding

        if not (self.shard_params and self.world >= 2):
            return [], []
        for m in self.module.modules():
            if isinstance(m, NgramEmbedding) and m.row_source is None:
                params = [t.weight for t in m.tables]
                if params and all(p.requires_grad and id(p) not in muon_ids for p in params):
                    return params, list(m.orders)
        return [], []

    def _allocate(self) -> None:
        dev = self.info.device
        if self.cuda:
            import torch.distributed._symmetric_memory as symm

            group = dist.group.WORLD
            self.flat_param = symm.empty(self.param_total, dtype=torch.float32, device=dev)
            self.flat_grad = symm.empty(self.grad_total, dtype=torch.float32, device=dev)
            self.flat_bf16 = symm.empty(self.bf16_total, dtype=torch.bfloat16, device=dev)
            self.ctrl = symm.empty(64, dtype=torch.int32, device=dev)  # [0, world): barrier flags; [32]: norm partial
            self.flat_mx = symm.empty(max(self.mx_total, 512), dtype=torch.uint8, device=dev)
            self.flat_grad.zero_()
            self.ctrl.zero_()
            handles = [symm.rendezvous(t, group) for t in (self.flat_param, self.flat_grad, self.flat_bf16, self.ctrl)]
            self._mx_handle = symm.rendezvous(self.flat_mx, group)
            self.mx_bases = torch.tensor(list(self._mx_handle.buffer_ptrs), dtype=torch.int64)  # host side
            ptrs = [torch.tensor(list(h.buffer_ptrs), dtype=torch.int64, device=dev) for h in handles]
            self.param_ptrs, self.grad_ptrs, self.bf16_ptrs, self.flag_ptrs = ptrs
            self.partial_ptrs = self.flag_ptrs + 32 * 4
            self.partial = self.ctrl[32:33].view(torch.float32)
            self._handles = handles
            self.grad_mc = self._multicast_address(handles[1], self.flat_grad)
        else:
            self.flat_param = torch.zeros(self.param_total, dtype=torch.float32, device=dev)
            self.flat_grad = torch.zeros(self.grad_total, dtype=torch.float32, device=dev)
            self.flat_bf16 = torch.zeros(self.bf16_total, dtype=torch.bfloat16, device=dev)

    def _multicast_address(self, handle, tensor: torch.Tensor) -> int:
        """NVSwitch multicast address of a symmetric buffer, or 0: with an address the gradient
        reduce-scatter reads through the switch (``multimem.ld_reduce``) instead of from
        every peer.  ``MYKB_NVLS``: ``0`` never, ``1`` whenever every rank's GPU supports
        NVLS, unset: only from 8 ranks.  A multicast read also carries the reading GPU's own
        copy over NVLink, N / (N - 1) times the bytes of the peer loads: measured on the
        200M gradient buffer the peer loads took 1.25 ms and the multicast read 2.42 ms at
        2 ranks, 2.52 ms and 2.27 ms at 8 ranks
        (``python -m myk_llm_b200.parallel.benchmark_collectives``)."""
        import os

        from torch._C._autograd import DeviceType
        from torch._C._distributed_c10d import _SymmetricMemory

        mode = os.environ.get("MYKB_NVLS", "auto")
        want = mode == "1" or (mode != "0" and self.world >= 8)
        ok = want and _SymmetricMemory.has_multicast_support(DeviceType.CUDA, tensor.device.index)
        mc = int(handle.multicast_ptr) if ok else 0
        flag = torch.tensor([1 if mc else 0], dtype=torch.int32, device=tensor.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)  # all ranks take the same path
        if not int(flag):
            return 0
        delta = tensor.data_ptr() - int(handle.buffer_ptrs[self.rank])
        return mc + delta

    def _load_params_into_buffers(self) -> None:
        """Copy the (identical on every rank after the broadcast) initial values into the
        flat buffers and point the parameters at them: views for replicated parameters, a
        one-element placeholder of the full shape for row-sharded ones."""
        dev = self.info.device
        rings: dict[tuple[int, int], list[GatherBuffer]] = {}
        count: dict[tuple[int, int], int] = {}
        with torch.no_grad():
            for s in self.slots:
                p = s.param
                full = p.detach().float()
                if dist.is_initialized():
                    full = full.contiguous()
                    dist.broadcast(full, src=0)
                g = self.flat_grad[s.goff:s.goff + s.numel].view_as(p)
                if not s.sharded:
                    view = self.flat_param[s.poff:s.poff + s.numel].view_as(p)
                    view.copy_(full)
                    p.data = view
                else:
                    lo = self.rank * s.rows_per_rank
                    hi = min(s.rows, lo + s.rows_per_rank)
                    shard = self.flat_param[s.poff:s.poff + s.shard_numel].view(s.rows_per_rank, s.cols)
                    shard.zero_()
                    if hi > lo:
                        shard[:hi - lo].copy_(full[lo:hi])
                    self.flat_bf16[s.boff:s.boff + s.shard_numel].copy_(shard.reshape(-1))
                    buf = None
                    if self.cuda:
                        key = (s.rows, s.cols)
                        if self.reshard_after_forward:
                            ring = rings.setdefault(key, [])
                            i = count.get(key, 0)
                            count[key] = i + 1
                            if len(ring) < 2:
                                ring.append(GatherBuffer(s.rows, s.cols, dev))
                            buf = ring[i % 2]
                        else:
                            buf = GatherBuffer(s.rows, s.cols, dev)
                    s.weight = ShardedWeight(self, s, buf)
                    p.data = torch.zeros(1, dtype=torch.float32, device=dev).expand(s.rows, s.cols)
                    p._mykb_shard = s.weight
                p.main_grad = g
                p.grad = g
        if self.cuda:
            torch.cuda.synchronize(dev)
            dist.barrier()

    def _build_ownership(self, optimizers, Muon, lr_ratio) -> None:
        by_param = {id(s.param): s for s in self.slots}
        self.muon_buckets: dict[tuple, dict] = {}
        adam_slots: list[tuple[Slot, dict]] = []
        for opt in optimizers:
            for group in opt.param_groups:
                for p in group["params"]:
                    if id(p) in self.table_ids:
                        self.tables.group = group
                        continue
                    s = by_param[id(p)]
                    if isinstance(opt, Muon):
                        key = (tuple(p.shape), s.sharded, s.rows_per_rank)  # one shard layout per bucket
                        b = self.muon_buckets.setdefault(key, {"slots": [], "group": group,
                                                               "ratio": lr_ratio(p.shape, group["adjust_lr"])})
                        b["slots"].append(s)
                    else:
                        adam_slots.append((s, group))
        # Muon: whole matrices, round-robin inside each bucket
        self.owned_muon = {key: [s for i, s in enumerate(b["slots"]) if i % self.world == self.rank]
                           for key, b in self.muon_buckets.items()}
        # AdamW: even slices of the concatenated AdamW index space (multiples of 4 elements);
        # AdamW parameters are always replicated, so gradient and parameter offsets agree
        self.adam_ranges: list[tuple[int, int, dict]] = []
        spans, acc = [], 0
        for s, g in adam_slots:
            n4 = _align(s.numel)
            spans.append((acc, s, g, n4))
            acc += n4
        per = (acc // self.world + 3) // 4 * 4
        lo = min(acc, self.rank * per)
        hi = min(acc, (self.rank + 1) * per) if self.rank < self.world - 1 else acc
        for start, s, g, n4 in spans:
            a, b_ = max(lo, start), min(hi, start + n4)
            if a < b_:
                self.adam_ranges.append((s.goff + (a - start), b_ - a, g))
        self._build_tables()
        dev = self.info.device
        n_adam = sum(r[1] for r in self.adam_ranges)
        self.adam_m = torch.zeros(n_adam, dtype=torch.float32, device=dev)
        self.adam_v = torch.zeros(n_adam, dtype=torch.float32, device=dev)
        self.muon_mom = {key: torch.zeros(len(sl), *key[0], dtype=torch.float32, device=dev)
                         for key, sl in self.owned_muon.items()}

    def _build_tables(self) -> None:
        dev = self.info.device

        def i64(xs):
            return torch.tensor(list(xs) or [0], dtype=torch.int64, device=dev)

        owned = [(s.goff, _align(s.numel)) for sl in self.owned_muon.values() for s in sl]
        owned += [(o, n) for o, n, _ in self.adam_ranges]
        owned.sort()
        pre = [0]
        for _, n in owned:
            pre.append(pre[-1] + n)
        self.red_offsets, self.red_prefix, self.red_total = i64(o for o, _ in owned)[:len(owned)], i64(pre), pre[-1]
        ap = [0]
        for _, n, _ in self.adam_ranges:
            ap.append(ap[-1] + n)
        self.adam_offsets, self.adam_prefix, self.adam_total = (i64(o for o, _, _ in self.adam_ranges),
                                                                i64(ap), ap[-1])
        self.muon_goffs = {key: i64(s.goff for s in sl) for key, sl in self.owned_muon.items()}
        self.muon_poffs = {key: i64(s.poff for s in sl) for key, sl in self.owned_muon.items()}
        self.muon_boffs = {key: i64(s.boff for s in sl) for key, sl in self.owned_muon.items()}
        # AdamW hyper-parameters per owned range, copied once; refreshed when they change
        self._adam_hp_key = None
        # set-up of the bf16 shards after a checkpoint load: (fp32 offset, length) -> bf16 offset
        shards = [s for s in self.slots if s.sharded]
        cp = [0]
        for s in shards:
            cp.append(cp[-1] + s.shard_numel)
        self.cast_src, self.cast_prefix, self.cast_dst, self.cast_total = (
            i64(s.poff for s in shards), i64(cp), i64(s.boff for s in shards), cp[-1])

    def _adam_hparams(self):
        from ..train.optim import Muon

        adam = [o for o in self.optimizers if not isinstance(o, Muon)]
        if not adam:
            return 0.9, 0.95, 1e-8
        g0 = adam[-1].param_groups[0]
        b1, b2 = g0["betas"]
        return b1, b2, g0["eps"]

    def _adam_lr_wd(self):
        """Per-range lr / weight decay on the device, re-uploaded only when a schedule changed them."""
        lr = [g["lr"] for _, _, g in self.adam_ranges] or [0.0]
        wd = [g["weight_decay"] for _, _, g in self.adam_ranges] or [0.0]
        key = (tuple(lr), tuple(wd))
        if key != self._adam_hp_key:
            dev = self.info.device
            self._adam_lr = torch.tensor(lr, dtype=torch.float32).pin_memory().to(dev, non_blocking=True) \
                if self.cuda else torch.tensor(lr)
            self._adam_wd = torch.tensor(wd, dtype=torch.float32).pin_memory().to(dev, non_blocking=True) \
                if self.cuda else torch.tensor(wd)
            self._adam_hp_key = key
        return self._adam_lr, self._adam_wd

    # -- the optimizer step ------------------------------------------------------------
    def _barrier(self) -> None:
        self.epoch += 1
        if self.cuda:
            ops.ext().peer_barrier(self.flag_ptrs, self.rank, self.world, self.epoch)

    @torch.no_grad()
    def optimizer_step(self, grad_clip: float) -> torch.Tensor:
        self.step_count += 1
        norm = self._step_cuda(grad_clip) if self.cuda else self._step_reference(grad_clip)
        self.version += 1
        self.trace.end_step()
        return norm

    def _step_cuda(self, grad_clip: float) -> torch.Tensor:
        ext = ops.ext()
        self.partial.zero_()
        self._barrier()
        if self.grad_mc:
            ext.dp_reduce_sumsq_multimem(self.grad_mc, self.flat_grad, self.red_offsets, self.red_prefix, self.partial,
                                         self.red_total)
        else:
            ext.dp_reduce_sumsq(self.grad_ptrs, self.rank, self.world, self.red_offsets, self.red_prefix,
                                self.partial, self.red_total)
        if self.tables is not None:
            self.tables.add_sumsq(self.partial)
        self._barrier()
        b1, b2, eps = self._adam_hparams()
        dev = self.info.device
        lr, wd = self._adam_lr_wd()
        norm = torch.zeros(1, dtype=torch.float32, device=dev)
        clip = float(grad_clip or 0.0)
        ext.dp_adamw_allgather(self.param_ptrs, self.grad_ptrs, self.rank, self.world, self.adam_offsets,
                               self.adam_prefix, wd, lr, self.adam_m, self.adam_v, b1, b2, eps, self.step_count,
                               self.partial_ptrs, 0.0, clip, norm, self.adam_total)
        if self.tables is not None:
            self.tables.adamw(self.step_count, b1, b2, eps, clip)
        for key, sl in self.owned_muon.items():
            if not sl:
                continue
            shape, sharded = key[:2]
            b = self.muon_buckets[key]
            g = b["group"]
            packed = torch.empty(len(sl), *shape, dtype=torch.bfloat16, device=dev)
            ext.dp_muon_prepare(self.grad_ptrs, self.rank, self.world, self.muon_goffs[key], math.prod(shape),
                                self.muon_mom[key], g["momentum"], g["nesterov"], packed, self.partial_ptrs, 0.0, clip)
            orth = ops.batched_newton_schulz_orthogonalize(packed, g["ns_steps"])
            decay, scale = g["lr"] * g["weight_decay"], -g["lr"] * b["ratio"]
            if sharded:
                ext.dp_muon_apply_shards(self.param_ptrs, self.bf16_ptrs, self.muon_poffs[key], self.muon_boffs[key],
                                         shape[0], shape[1], sl[0].rows_per_rank, decay, scale, orth.contiguous())
            else:
                ext.dp_muon_apply_allgather(self.param_ptrs, self.rank, self.world, self.muon_poffs[key],
                                            math.prod(shape), decay, scale, orth)
        self._barrier()
        self._quantize_mx_shards()  # the new rows' fp8 copies (own barrier)
        # A peer wait that gave up leaves its code in the device status word; the trainer
        # reads it at its next host sync (Trainer.check_health).
        self.last_norm = norm[0]
        return norm[0]

    def gather_full_fp32(self, s: Slot) -> torch.Tensor:
        """The full fp32 master of a row-sharded weight (collective over all ranks)."""
        mine = self.flat_param[s.poff:s.poff + s.shard_numel].view(s.rows_per_rank, s.cols)
        if not dist.is_initialized():
            return mine[:s.rows].clone()
        parts = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(parts, mine.contiguous())
        return torch.cat(parts, 0)[:s.rows]

    def _set_full_fp32(self, s: Slot, full: torch.Tensor) -> None:
        """Write this rank's rows of a full fp32 weight into its master and bf16 shards."""
        lo = self.rank * s.rows_per_rank
        hi = min(s.rows, lo + s.rows_per_rank)
        shard = self.flat_param[s.poff:s.poff + s.shard_numel].view(s.rows_per_rank, s.cols)
        shard.zero_()
        if hi > lo:
            shard[:hi - lo].copy_(full[lo:hi].to(shard.dtype))
        self.flat_bf16[s.boff:s.boff + s.shard_numel].copy_(shard.reshape(-1))

    def _step_reference(self, grad_clip: float) -> torch.Tensor:
        """CPU / gloo path with the same ownership and arithmetic (all_reduce based)."""
        if dist.is_initialized():
            dist.all_reduce(self.flat_grad)
        sq = torch.zeros((), dtype=torch.float64)
        sizes = (self.red_prefix[1:] - self.red_prefix[:-1]).tolist()
        for o, n in zip(self.red_offsets.tolist(), sizes):
            sq += self.flat_grad[o:o + n].double().square().sum()
        if self.tables is not None:  # this rank's table rows (each row is owned by one rank)
            sq += self.tables.grad.double().square().sum()
        if dist.is_initialized():
            dist.all_reduce(sq)
        norm = sq.sqrt().float()
        coef = min(1.0, grad_clip / (float(norm) + 1e-6)) if grad_clip and grad_clip > 0 else 1.0
        b1, b2, eps = self._adam_hparams()
        if self.tables is not None:
            self.tables.step_cpu(self.step_count, b1, b2, eps, coef)
        bc1 = 1 - b1 ** self.step_count
        bc2 = math.sqrt(1 - b2 ** self.step_count)
        new = torch.zeros(self.rep_total)
        mask = torch.zeros(self.rep_total, dtype=torch.bool)
        pos = 0
        for o, n, g in self.adam_ranges:
            p = self.flat_param[o:o + n]
            gr = self.flat_grad[o:o + n] * coef
            m, v = self.adam_m[pos:pos + n], self.adam_v[pos:pos + n]
            m.lerp_(gr, 1 - b1)
            v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
            new[o:o + n] = p * (1 - g["lr"] * g["weight_decay"]) - (g["lr"] / bc1) * m / (v.sqrt() / bc2 + eps)
            mask[o:o + n] = True
            pos += n
        shard_updates: dict[int, torch.Tensor] = {}
        for key, b in self.muon_buckets.items():
            shape, sharded = key[:2]
            g = b["group"]
            mine = self.owned_muon[key]
            ups = []
            for i, s in enumerate(mine):
                gr = self.flat_grad[s.goff:s.goff + s.numel].view(shape) * coef
                self.muon_mom[key][i].lerp_(gr, 1 - g["momentum"])
                mom = self.muon_mom[key][i]
                ups.append(gr.lerp(mom, g["momentum"]) if g["nesterov"] else mom.clone())
            orth = newton_schulz_ref(torch.stack(ups), g["ns_steps"]) if ups else None
            decay, scale = g["lr"] * g["weight_decay"], -g["lr"] * b["ratio"]
            for s in b["slots"]:  # every rank walks every matrix of the bucket (collectives inside)
                full = s.weight.full_cpu() if sharded else self.flat_param[s.poff:s.poff + s.numel].view(shape)
                i = next((j for j, t in enumerate(mine) if t is s), None)
                if sharded:
                    upd = torch.zeros(shape)
                    if i is not None:
                        upd = full * (1 - decay) + scale * orth[i].float()
                    shard_updates[id(s)] = upd
                elif i is not None:
                    new[s.poff:s.poff + s.numel] = (full * (1 - decay) + scale * orth[i].float()).reshape(-1)
                    mask[s.poff:s.poff + s.numel] = True
        contrib = torch.where(mask, new, torch.zeros_like(new))
        rep = self.flat_param[:self.rep_total]
        if dist.is_initialized():
            dist.all_reduce(contrib)
            owned_any = mask.float()
            dist.all_reduce(owned_any)
            rep.copy_(torch.where(owned_any > 0, contrib, rep))
        else:
            rep.copy_(torch.where(mask, contrib, rep))
        for s in self.slots:
            if s.sharded:
                upd = shard_updates[id(s)]
                if dist.is_initialized():
                    dist.all_reduce(upd)  # exactly one rank (the owner) contributed
                self._set_full_fp32(s, upd)
        self.last_norm = norm
        return norm

    # -- checkpoint plumbing -----------------------------------------------------------
    def sync_params_for_checkpoint(self) -> None:
        """Before a DCP save: materialise full per-parameter optimizer state (Muon
        momentum_buffer, AdamW step/exp_avg/exp_avg_sq) in the torch optimizers, and full fp32
        values for row-sharded weights, so the checkpoint has the reference's layout."""
        from ..train.optim import Muon

        dev = self.info.device
        full_m = torch.zeros(self.grad_total, dtype=torch.float32, device=dev)
        full_v = torch.zeros_like(full_m)
        full_mom = torch.zeros_like(full_m)
        pos = 0
        for o, n, _ in self.adam_ranges:
            full_m[o:o + n] = self.adam_m[pos:pos + n]
            full_v[o:o + n] = self.adam_v[pos:pos + n]
            pos += n
        for key, sl in self.owned_muon.items():
            for i, s in enumerate(sl):
                full_mom[s.goff:s.goff + s.numel] = self.muon_mom[key][i].reshape(-1)
        if dist.is_initialized():
            for t in (full_m, full_v, full_mom):
                dist.all_reduce(t)
        slot_of = {id(s.param): s for s in self.slots}
        table_index = {id(p): j for j, p in enumerate(self.tables.params)} if self.tables is not None else {}
        for opt in self.optimizers:
            for group in opt.param_groups:
                for p in group["params"]:
                    if id(p) in table_index:  # row-sharded table: gather its moments (collective)
                        j, st = table_index[id(p)], opt.state[p]
                        st["step"] = torch.tensor(float(self.step_count))
                        st["exp_avg"] = self.tables.gather(self.tables.m, j)
                        st["exp_avg_sq"] = self.tables.gather(self.tables.v, j)
                        continue
                    s = slot_of[id(p)]
                    st = opt.state[p]
                    sl = slice(s.goff, s.goff + s.numel)
                    if isinstance(opt, Muon):
                        st["momentum_buffer"] = full_mom[sl].view(p.shape).clone()
                    else:
                        st["step"] = torch.tensor(float(self.step_count))
                        st["exp_avg"] = full_m[sl].view(p.shape).clone()
                        st["exp_avg_sq"] = full_v[sl].view(p.shape).clone()
        self._materialise_sharded()

    def _materialise_sharded(self) -> None:
        with torch.no_grad():
            for s in self.slots:
                if s.sharded:
                    s.param.data = self.gather_full_fp32(s).contiguous()
        if self.tables is not None:
            self.tables.materialise()

    def _dematerialise_sharded(self) -> None:
        dev = self.info.device
        for s in self.slots:
            if s.sharded:
                s.param.data = torch.zeros(1, dtype=torch.float32, device=dev).expand(s.rows, s.cols)
        if self.tables is not None:
            self.tables.dematerialise()

    def after_checkpoint_save(self) -> None:
        self._dematerialise_sharded()

    def before_checkpoint_load(self) -> None:
        """DCP loads in place into the tensors of the current state: give row-sharded
        parameters full-size storage, and the torch optimizers full per-parameter state
        (the gradients are the runtime's buffers, so torch cannot create that state with a
        trial step)."""
        self.sync_params_for_checkpoint()

    def after_checkpoint_load(self) -> None:
        """Scatter loaded values and per-parameter optimizer state back into the shards."""
        from ..train.optim import Muon

        with torch.no_grad():
            for s in self.slots:
                if s.sharded and s.param.data.stride() != (0, 0):
                    self._set_full_fp32(s, s.param.data)
            if self.tables is not None:
                for j, p in enumerate(self.tables.params):
                    if p.data.stride() != (0, 0):
                        self.tables.scatter(self.tables.param, j, p.data)
            self._dematerialise_sharded()
        slot_of = {id(s.param): s for s in self.slots}
        dev = self.info.device
        flat_m = torch.zeros(self.grad_total, dtype=torch.float32, device=dev)
        flat_v = torch.zeros_like(flat_m)
        flat_mom = torch.zeros_like(flat_m)
        step = None
        table_index = {id(p): j for j, p in enumerate(self.tables.params)} if self.tables is not None else {}
        for opt in self.optimizers:
            for group in opt.param_groups:
                for p in group["params"]:
                    if id(p) in table_index:
                        st = opt.state.get(p, {})
                        if "exp_avg" in st:
                            j = table_index[id(p)]
                            self.tables.scatter(self.tables.m, j, st["exp_avg"].float())
                            self.tables.scatter(self.tables.v, j, st["exp_avg_sq"].float())
                            step = int(float(st["step"]))
                        continue
                    s = slot_of[id(p)]
                    st = opt.state.get(p, {})
                    sl = slice(s.goff, s.goff + s.numel)
                    if isinstance(opt, Muon) and "momentum_buffer" in st:
                        flat_mom[sl] = st["momentum_buffer"].reshape(-1).float()
                    elif "exp_avg" in st:
                        flat_m[sl] = st["exp_avg"].reshape(-1).float()
                        flat_v[sl] = st["exp_avg_sq"].reshape(-1).float()
                        step = int(float(st["step"]))
        pos = 0
        for o, n, _ in self.adam_ranges:
            self.adam_m[pos:pos + n] = flat_m[o:o + n]
            self.adam_v[pos:pos + n] = flat_v[o:o + n]
            pos += n
        for key, sl in self.owned_muon.items():
            for i, s in enumerate(sl):
                self.muon_mom[key][i].copy_(flat_mom[s.goff:s.goff + s.numel].view(key[0]))
        if step is not None:
            self.step_count = step
        self.version += 1
        if self.cuda:
            torch.cuda.synchronize(dev)
            dist.barrier()
            self._quantize_mx_shards(sync=True)

    def full_named_parameters(self) -> dict[str, torch.Tensor]:
        """Every trainable parameter as a full fp32 tensor (row-sharded weights gathered: a
        collective, so every rank calls it)."""
        out = {}
        table_index = {id(p): j for j, p in enumerate(self.tables.params)} if self.tables is not None else {}
        for n, p in self.module.named_parameters():
            s = getattr(p, "_mykb_shard", None)
            if id(p) in table_index:
                out[n] = self.tables.gather(self.tables.param, table_index[id(p)])
            else:
                out[n] = self.gather_full_fp32(s.slot).clone() if s is not None else p.detach().clone()
        return out

    # -- memory report ------------------------------------------------------------------
    def memory_bytes(self) -> dict[str, int]:
        """Bytes this rank holds for parameters, gradients, optimizer state and gather buffers."""
        bufs = {id(s.weight.buf): s.weight.buf for s in self.slots if s.sharded and s.weight.buf is not None}
        return {
            "params_fp32": self.flat_param.numel() * 4,
            "params_bf16_shards": self.flat_bf16.numel() * 2,
            "grads_fp32": self.flat_grad.numel() * 4,
            "optimizer_state": (self.adam_m.numel() + self.adam_v.numel()
                                + sum(t.numel() for t in self.muon_mom.values())) * 4,
            "gather_buffers": sum(b.w.numel() * 2 for b in bufs.values()),
            "ngram_table_shards": self.tables.memory_bytes() if self.tables is not None else 0,
        }


def shard_model(model: nn.Module, info: DistInfo, reshard_after_forward: bool = True,
                shard_params: bool = True) -> ShardedDataParallel:
    return ShardedDataParallel(model, info, shard_params=shard_params, reshard_after_forward=reshard_after_forward)
