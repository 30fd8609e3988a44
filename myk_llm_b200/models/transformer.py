"""The MykLLM decoder: embeddings -> blocks -> final norm (+ MTP modules).

Behaviour follows the reference model (``src/myk_llm/model/transformer.py:56-417``):
pre-norm sequential or parallel blocks with residual gates, DeepSeek-V3 MTP modules, a
looped core with add/concat injection and truncated backpropagation, the YOCO
decoder-decoder (shared KV, cross blocks, ``keep_last``), n-gram injection per block,
document masking through ``seqlens``, and a ``head`` callback so losses run inside
forward.  The cache is a list with one entry per self-decoder block call, plus the shared
KV, plus one empty entry per cross block.

Differences in mechanism, not in results: there is no ``torch.compile``; blocks call the
fused sm_100a kernels directly.  With an ungated residual the residual add and the next
RMSNorm run as one kernel (``ops.add_rms_norm``).
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Callable

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .. import ops
from .config import GLOBAL_ATTENTION, ModelConfig
from .embeddings import Embeddings
from .layers import ResidualGate, RMSNorm, SwiGLU, init_linear_, residual_init_scale
from .mixers import Attention, SharedKV, Varlen, build_mixer

_side_streams: dict[int, torch.cuda.Stream] = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    idx = torch.cuda.current_device() if device.index is None else device.index
    if idx not in _side_streams:
        _side_streams[idx] = torch.cuda.Stream(idx)
    return _side_streams[idx]


def _concurrently(first: Callable[[], Any], second: Callable[[], Any], side: torch.cuda.Stream):
    """Run first() on the current stream and second() on ``side``; join afterwards."""
    main = torch.cuda.current_stream()
    side.wait_stream(main)
    with torch.cuda.stream(side):
        b = second()
    a = first()
    main.wait_stream(side)
    return a, b


@dataclass
class PendingResidual:
    """A residual-stream value kept as ``base + delta`` (the block's fp32 stream and its last
    FFN output): the next block's pre-norm (or the final norm) adds and normalises in one
    kernel instead of an add pass followed by a norm pass."""

    base: torch.Tensor
    delta: torch.Tensor


def materialize(x):
    return x.base + x.delta if isinstance(x, PendingResidual) else x


# a pytree node, so wrappers that walk module outputs (FSDP2 hooks) see both tensors
torch.utils._pytree.register_pytree_node(
    PendingResidual, lambda r: ([r.base, r.delta], None), lambda xs, _: PendingResidual(*xs),
    serialized_type_name="myk_llm_b200.PendingResidual")


class Block(nn.Module):
    """x + g1*mixer(norm(x)) then + g2*ffn(norm(x)); or parallel: x + g1*mixer(h) + g2*ffn(h)."""

    def __init__(self, config: ModelConfig, layer_type: str, first_global: bool) -> None:
        super().__init__()
        self.layer_type = layer_type
        self.mixer_norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.mixer = build_mixer(config, layer_type, first_global)
        self.mixer_gate = ResidualGate(config.residual, config.hidden_size)
        self.ffn_norm = None if config.parallel_block else RMSNorm(config.hidden_size, config.norm_eps)
        self.ffn = SwiGLU(config)
        self.ffn_gate = ResidualGate(config.residual, config.hidden_size)
        self.streams = config.parallel_streams
        self.activation_checkpointing = False
        # set by MykLLM for its main stack: return PendingResidual instead of adding the FFN
        # output here (the consumer fuses the add with its norm)
        self.defer_residual = False

    def residual_projections(self) -> list[nn.Linear]:
        return [*self.mixer.residual_projections(), self.ffn.down_proj]

    def forward(self, x, position_ids, varlen: Varlen | None = None, state: Any = None, use_cache: bool = False):
        if self.activation_checkpointing and torch.is_grad_enabled() and not use_cache:
            return checkpoint(Block._forward, self, x, position_ids, varlen, state, False, use_reentrant=False)
        return self._forward(x, position_ids, varlen, state, use_cache)

    def _enter(self, x):
        """(residual stream, normed mixer input): a pending FFN output from the previous
        block is added here, in the same kernel as this block's pre-norm."""
        if isinstance(x, PendingResidual):
            return ops.add_rms_norm(x.base, x.delta, self.mixer_norm.weight, self.mixer_norm.eps,
                                    out_dtype=ops.compute_dtype(x.base))
        return x, self.mixer_norm(x, out_dtype=ops.compute_dtype(x))

    def _forward(self, x, position_ids, varlen, state, use_cache):
        x, h = self._enter(x)
        if self.ffn_norm is None:  # parallel block: one norm, both branches read it
            (update, state), f = self._parallel(h, position_ids, varlen, state, use_cache)
            return self.ffn_gate(self.mixer_gate(x, update, h), f, h), state
        update, state = self.mixer(h, position_ids, varlen, state, use_cache)
        if self.mixer_gate.kind == "none":  # residual add fused with the FFN pre-norm
            x, h = ops.add_rms_norm(x, update, self.ffn_norm.weight, self.ffn_norm.eps, out_dtype=h.dtype)
        else:
            x = self.mixer_gate(x, update, h)
            h = self.ffn_norm(x, out_dtype=ops.compute_dtype(x))
        f = self.ffn(h)
        if self.defer_residual and self.ffn_gate.kind == "none":
            return PendingResidual(x, f), state  # the next norm adds it
        return self.ffn_gate(x, f, h), state

    def side_stream(self, device: torch.device) -> torch.cuda.Stream:
        s = self.__dict__.get("_side_stream")
        if s is None:
            s = self.__dict__["_side_stream"] = _side_stream(device)
        return s

    def _parallel(self, h, position_ids, varlen, state, use_cache):
        def mixer():
            return self.mixer(h, position_ids, varlen, state, use_cache)

        def ffn():
            return self.ffn(h)

        if self.streams and h.is_cuda and not torch.is_grad_enabled():
            return _concurrently(mixer, ffn, self.side_stream(h.device))
        return mixer(), ffn()


class MTPModule(nn.Module):
    """proj([norm(h), norm(emb(t+k))]) -> one block; ``final_norm`` feeds the shared head."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.hidden_norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.embed_norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.proj = nn.Linear(2 * config.hidden_size, config.hidden_size, bias=False)
        self.block = Block(config, config.mtp.layer, first_global=True)
        self.final_norm = RMSNorm(config.hidden_size, config.norm_eps)

    def forward(self, hidden, next_embed, position_ids, varlen, state: Any = None, use_cache: bool = False):
        cdt = ops.compute_dtype(hidden)
        cat = torch.cat([self.hidden_norm(hidden, out_dtype=cdt), self.embed_norm(next_embed, out_dtype=cdt)], dim=-1)
        x = ops.linear(cat, self.proj.weight)
        if cdt != hidden.dtype:
            x = x.to(hidden.dtype)
        x, state = self.block(x, position_ids, varlen, state, use_cache)
        return (x, state) if use_cache else x


class Injection(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.kind = config.loop.injection
        if self.kind == "concat":
            self.state_norm = RMSNorm(config.hidden_size, config.norm_eps)
            self.input_norm = RMSNorm(config.hidden_size, config.norm_eps)
            self.proj = nn.Linear(2 * config.hidden_size, config.hidden_size, bias=False)

    def forward(self, state, inputs):
        if self.kind == "add":
            return state + inputs
        cdt = ops.compute_dtype(state)
        cat = torch.cat([self.state_norm(state, out_dtype=cdt), self.input_norm(inputs, out_dtype=cdt)], -1)
        return ops.linear(cat, self.proj.weight).to(state.dtype)


@dataclass
class ModelOutput:
    hidden: torch.Tensor
    residual: torch.Tensor
    position_ids: torch.Tensor
    varlen: Varlen | None
    cache: list[Any] | None = None


_NVTX = [False]


def set_nvtx(enabled: bool) -> None:
    """Emit NVTX ranges (per layer here, per training phase in the trainer) for timeline
    profilers; off by default (no cost when off)."""
    _NVTX[0] = bool(enabled)


class nvtx_range:
    """``with nvtx_range(name):`` pushes an NVTX range when enabled and on a CUDA build."""

    def __init__(self, name: str) -> None:
        self.name = name
        self.on = _NVTX[0] and torch.cuda.is_available()

    def __enter__(self):
        if self.on:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if self.on:
            torch.cuda.nvtx.range_pop()
        return False


def build_varlen(seqlens: list[torch.Tensor], batch: int, seq_len: int, device: torch.device) -> Varlen:
    lengths = torch.cat([s.to(device="cpu", dtype=torch.int32) for s in seqlens])
    cu_cpu = F.pad(lengths.cumsum(0, dtype=torch.int32), (1, 0))
    if device.type == "cuda":
        cu_cpu = cu_cpu.pin_memory()
    cu = cu_cpu.to(device=device, non_blocking=True)
    return Varlen(cu_seqlens=cu, max_seqlen=seq_len, cu_seqlens_cpu=cu_cpu)


class _Pass:
    """One forward pass's walk over the blocks.

    Cache layout (what ``use_cache`` returns and ``cache`` must match): one entry per
    self-decoder block call in execution order (the looped core contributes one entry per
    block per iteration), then the projected shared KV (``cross.kv = project``), then one
    empty entry per cross-decoder block.  The cross-decoder reads the shared KV (projected,
    or the state of block ``cross_kv_layer``) and keeps no state of its own.
    """

    def __init__(self, model: "MykLLM", positions, varlen, cache, use_cache: bool, injections: dict, iterations: int):
        cfg = model.config
        self.model, self.positions, self.varlen, self.use_cache = model, positions, varlen, use_cache
        self.injections, self.iterations, self.loop = injections, iterations, cfg.loop
        n, start = len(model.layers), model.cross_start
        self.has_cross = start < n
        # a loop whose core lies in the cross-decoder repeats stateless cross blocks only
        self.core_in_cross = bool(self.loop.core) and self.loop.prelude >= start
        repeated = 0 if self.core_in_cross else self.loop.core * (iterations - 1)
        calls = n + repeated + (model.shared_kv is not None)
        if cache is not None and len(cache) != calls:
            raise ValueError(f"cache has {len(cache)} entries but this pass runs {calls} blocks "
                             "(iteration count changed?)")
        self.states = iter(cache) if cache is not None else None
        self.new_cache: list[Any] | None = [] if use_cache else None
        self.shared: Any = None

    def _state(self):
        return next(self.states) if self.states is not None else None

    def _keep(self, state) -> None:
        if self.new_cache is not None:
            self.new_cache.append(state)

    def _inject(self, i: int, x):
        update = self.injections.get(i)
        if update is None:
            return x
        x = materialize(x)
        return x + update[:, -x.shape[1]:]

    def self_block(self, i: int, x):
        with nvtx_range(f"layer{i}"):
            x, state = self.model.layers[i](x, self.positions, self.varlen, self._state(), self.use_cache)
        self._keep(state)
        if i == self.model.cross_kv_layer:
            self.shared = state
        return x

    def cross_block(self, i: int, x):
        with nvtx_range(f"layer{i}"):
            return self.model.layers[i](x, self.positions, self.varlen, self.shared)[0]

    def _span(self, lo: int, hi: int, call, looped: bool, x):
        """Blocks [lo, hi) with n-gram injections; the loop core in it runs looped."""
        core_lo, core_hi = (self.loop.prelude, self.loop.prelude + self.loop.core) if looped else (hi, hi)
        for i in range(lo, core_lo):
            x = call(i, self._inject(i, x))
        if looped:
            x = self.model._run_core(materialize(self._inject(core_lo, x)), call, self.iterations)
        for i in range(core_hi, hi):
            x = call(i, self._inject(i, x))
        return x

    def self_decoder(self, x):
        looped = bool(self.loop.core) and not self.core_in_cross
        return self._span(0, self.model.cross_start, self.self_block, looped, x)

    def cross_decoder(self, x, keep_last: int):
        """Shared KV from the full self-decoder output, then the cross blocks on the last
        ``keep_last`` positions (all of them when 0)."""
        model = self.model
        full_x, full_pos = x, self.positions
        if model.shared_kv is not None:
            self.shared = model.shared_kv(full_x, full_pos, self._state())
            self._keep(self.shared)
        for _ in range(model.cross_start, len(model.layers)):
            self._state()
            self._keep(None)
        if keep_last:
            x, self.positions = x[:, -keep_last:], self.positions[:, -keep_last:]
        return self._span(model.cross_start, len(model.layers), self.cross_block, self.core_in_cross, x)


class MykLLM(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.embed = Embeddings(config)
        globals_ = [i for i, t in enumerate(config.layer_types) if t == GLOBAL_ATTENTION]
        first_global = globals_[0] if globals_ else -1
        self.layers = nn.ModuleList(Block(config, t, first_global=(i == first_global))
                                    for i, t in enumerate(config.layer_types))
        for block in self.layers:
            block.defer_residual = True
        self.final_norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_embeddings:
            self.lm_head.weight = self.embed.token.weight
        self.mtp = nn.ModuleList(MTPModule(config) for _ in range(config.mtp.depth))
        self.injection = Injection(config) if config.loop.core else None
        self.cross_start, self.cross_kv_layer = config.cross_start, config.cross_kv_layer
        has_cross = self.cross_start < len(self.layers)
        self.shared_kv = SharedKV(config) if has_cross and config.cross.kv == "project" else None
        if self.cross_kv_layer is not None:
            src = self.layers[self.cross_kv_layer].mixer
            assert isinstance(src, Attention)
            src.shares_kv = True
        self._iteration_rng = random.Random(torch.initial_seed())
        # analysis hook: called as fn(iteration, loop state) after every pass of a looped core
        self.core_observer: Callable[[int, torch.Tensor], None] | None = None
        self.init_weights()

    @torch.no_grad()
    def init_weights(self) -> None:
        std = self.config.initializer_range
        self.apply(lambda m: init_linear_(m, std))
        scale = residual_init_scale(self.config.effective_layers)
        for block in self.blocks:
            for proj in block.residual_projections():
                proj.weight.mul_(scale)
            block.mixer_gate.init_weights()
            block.ffn_gate.init_weights()

    @property
    def output_weight(self) -> torch.Tensor:
        return self.lm_head.weight

    @property
    def device(self) -> torch.device:
        return self.embed.token.weight.device

    def num_parameters(self, exclude_embeddings: bool = False) -> int:
        params = {id(p): p for p in self.parameters()}
        if exclude_embeddings:
            for p in [*self.embed.parameters(), self.lm_head.weight]:
                params.pop(id(p), None)
        return sum(p.numel() for p in params.values())

    @property
    def blocks(self) -> list[Block]:
        return [*self.layers, *(m.block for m in self.mtp)]

    def compile_blocks(self, **kwargs: Any) -> None:
        """Kept for API parity: blocks already run hand-written fused kernels, so there is
        nothing for a tracing compiler to do; decode loops use CUDA graphs instead."""
        return None

    def set_activation_checkpointing(self, enabled: bool | int) -> None:
        stride = (1 if enabled else 0) if isinstance(enabled, bool) else int(enabled)
        if stride < 0:
            raise ValueError(f"activation_checkpointing must be a bool or >= 0, got {enabled!r}")
        for i, block in enumerate(self.blocks):
            block.activation_checkpointing = bool(stride and i % stride == 0)

    def forward(self, input_ids, position_ids=None, seqlens=None, cache=None, use_cache=False, prefix_ids=None,
                head: Callable[["MykLLM", ModelOutput], Any] | None = None, embed_offset=None, iterations=None,
                keep_last: int = 0):
        bsz, seq = input_ids.shape
        if position_ids is None:
            position_ids = torch.arange(seq, device=input_ids.device).expand(bsz, -1)
        if seqlens is not None and (use_cache or keep_last):
            raise ValueError("document masking (seqlens) cannot be combined with a cache or keep_last")
        varlen = build_varlen(seqlens, bsz, seq, input_ids.device) if seqlens is not None else None
        x, injections = self.embed(input_ids, prefix_ids)
        if embed_offset is not None:
            x = x + embed_offset
        run = _Pass(self, position_ids, varlen, cache, use_cache, injections, self.num_iterations(iterations))
        x = run.self_decoder(x)
        if keep_last or run.has_cross:
            x = materialize(x)
        if run.has_cross:
            x = run.cross_decoder(x, keep_last)
        elif keep_last:
            x = x[:, -keep_last:]
        positions = position_ids[:, -keep_last:] if keep_last else position_ids
        if isinstance(x, PendingResidual):
            x, hidden = ops.add_rms_norm(x.base, x.delta, self.final_norm.weight, self.final_norm.eps,
                                         out_dtype=ops.compute_dtype(x.base))
        else:
            hidden = self.final_norm(x, out_dtype=ops.compute_dtype(x))
        out = ModelOutput(hidden, x, positions, varlen, run.new_cache)
        return head(self, out) if head is not None else out

    def num_iterations(self, iterations: int | None = None) -> int:
        loop = self.config.loop
        if not loop.core:
            if iterations is not None:
                raise ValueError("iterations needs a looped model (model.loop.core > 0)")
            return 1
        if iterations is not None:
            if iterations < 1:
                raise ValueError(f"iterations must be >= 1, got {iterations}")
            return iterations
        if self.training and loop.train_iterations:
            return self._iteration_rng.randint(*loop.train_iterations)
        return loop.iterations

    def _run_core(self, inputs, block, iterations):
        loop, inj = self.config.loop, self.injection
        assert inj is not None
        grad = torch.is_grad_enabled()
        first_tracked = iterations - loop.backprop_iterations if grad and loop.backprop_iterations else 0
        state = torch.zeros_like(inputs)
        for it in range(iterations):
            with torch.set_grad_enabled(grad and it >= first_tracked):
                state = inj(materialize(state), inputs)
                for i in range(loop.prelude, loop.prelude + loop.core):
                    state = block(i, state)
            if self.core_observer is not None:
                state = materialize(state)
                self.core_observer(it, state)
        return materialize(state)

    def cache_blocks(self, iterations: int | None = None) -> list[Any]:
        """What each entry of the decode cache belongs to, in the order ``forward`` consumes
        them (the ``_Pass`` layout): the block of every self-decoder call (a looped core's
        blocks once per iteration), ``"shared_kv"`` for the projected YOCO KV, and None for
        each cross-decoder block."""
        n, start, loop = len(self.layers), self.cross_start, self.config.loop
        order = list(range(start))
        if loop.core and loop.prelude < start:
            core = list(range(loop.prelude, loop.prelude + loop.core))
            order = list(range(loop.prelude)) + core * self.num_iterations(iterations) + \
                list(range(loop.prelude + loop.core, start))
        entries: list[Any] = [self.layers[i] for i in order]
        if self.shared_kv is not None:
            entries.append("shared_kv")
        return entries + [None] * (n - start)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return ops.linear(hidden, self.lm_head.weight)

    def mtp_hidden(self, output: ModelOutput, input_ids: torch.Tensor) -> list[torch.Tensor]:
        hidden, results = output.residual, []
        for k, module in enumerate(self.mtp, start=1):
            shifted = F.pad(input_ids[:, k:], (0, k), value=0)
            hidden = module(hidden, ops.embedding(shifted, self.embed.token.weight), output.position_ids, output.varlen)
            results.append(module.final_norm(hidden, out_dtype=ops.compute_dtype(hidden)))
        return results
