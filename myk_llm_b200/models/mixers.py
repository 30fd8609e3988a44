"""Token mixers: softmax attention (global / sliding window), YOCO shared KV and cross
attention, and Gated DeltaNet / Kimi Delta Attention.

Every mixer is called as ``mixer(x, position_ids, varlen, state, use_cache) ->
(out, new_state)`` (reference: ``src/myk_llm/model/mixers.py:1-12``).  ``varlen`` holds
packed-document boundaries for document-masked training; ``state`` is the mixer's own
decode cache (``KVCache`` / ``StaticKV`` for attention, ``DeltaState`` /
``SpecDeltaState`` for DeltaNet).  Cross-decoder mixers receive the shared KV as ``state``.

The parameter names are the reference's (which for DeltaNet are flash-linear-attention's
``GatedDeltaNet`` / ``KimiDeltaAttention`` names under ``mixer.inner``), so DCP
checkpoints and ``model.safetensors`` exports interchange.  The DeltaNet math here is
our own (:mod:`myk_llm_b200.ops.gdn`); flash-linear-attention is not used.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn

from .. import ops
from .config import CROSS_ATTENTION, DELTANET, GLOBAL_ATTENTION, LOCAL_ATTENTION, ModelConfig
from .layers import RMSNorm, RotaryEmbedding


@dataclass
class Varlen:
    """Packed-document layout of a (batch, seq_len) block flattened row-major."""

    cu_seqlens: torch.Tensor  # int32 (num_docs + 1,) on the compute device
    max_seqlen: int
    cu_seqlens_cpu: torch.Tensor | None = None


@dataclass
class KVCache:
    keys: torch.Tensor  # (batch, cached_len, kv_heads, head_dim)
    values: torch.Tensor


@dataclass
class StaticKV:
    """Preallocated decode cache of one attention layer: keys/values (batch, capacity,
    kv_heads, head_dim) and the per-row number of valid positions ``seqlens`` (int32, shared
    by all layers and advanced by the decoder).  New keys/values are written at
    ``seqlens[b]`` onward without host synchronisation, so a decode step can be captured
    in a CUDA graph."""

    keys: torch.Tensor
    values: torch.Tensor
    seqlens: torch.Tensor


class Attention(nn.Module):
    """Grouped-query causal softmax attention, global or sliding-window."""

    def __init__(self, config: ModelConfig, local: bool, use_rope: bool) -> None:
        super().__init__()
        a = config.attention
        self.num_heads, self.num_kv_heads, self.head_dim = a.num_heads, a.num_kv_heads, a.head_dim
        self.local = local
        self.window = a.sliding_window if local else None
        self.max_seq_len = config.max_seq_len
        qs, kvs = a.num_heads * a.head_dim, a.num_kv_heads * a.head_dim
        self.split = (qs, kvs, kvs)
        self.qkv_proj = nn.Linear(config.hidden_size, qs + 2 * kvs, bias=False)
        self.o_proj = nn.Linear(qs, config.hidden_size, bias=False)
        self.q_norm = RMSNorm(a.head_dim, config.norm_eps) if a.qk_norm else None
        self.k_norm = RMSNorm(a.head_dim, config.norm_eps) if a.qk_norm else None
        self.gate_proj = nn.Linear(config.hidden_size, qs, bias=False) if a.output_gate else None
        theta = a.rope_theta_local if local else a.rope_theta_global
        self.rope = RotaryEmbedding(a.head_dim, config.max_seq_len, theta) if use_rope else None
        self.shares_kv = False  # set when this layer is the source of a YOCO shared KV

    def residual_projections(self) -> list[nn.Linear]:
        return [self.o_proj]

    def forward(self, x, position_ids, varlen: Varlen | None = None, state: KVCache | None = None,
                use_cache: bool = False):
        bsz, seq, _ = x.shape
        qkv = ops.linear(x, self.qkv_proj.weight)
        if self.rope is not None and self.q_norm is None and qkv.is_cuda:
            q, k, v = self.rope.split_qkv(qkv, position_ids, self.num_heads, self.num_kv_heads)
        else:
            q, k, v = qkv.split(self.split, dim=-1)
            q = q.view(bsz, seq, self.num_heads, self.head_dim)
            k = k.view(bsz, seq, self.num_kv_heads, self.head_dim)
            v = v.view(bsz, seq, self.num_kv_heads, self.head_dim)
            if self.q_norm is not None and self.k_norm is not None:
                q = self.q_norm(q, out_dtype=v.dtype)
                k = self.k_norm(k, out_dtype=v.dtype)
            if self.rope is not None:
                q, k = self.rope(q, k, position_ids)
        window = (self.window - 1, 0) if self.window is not None else (-1, -1)
        new_state = KVCache(k, v) if self.shares_kv else None
        if isinstance(state, StaticKV):
            out = ops.flash_attn_with_kvcache(q, state.keys, state.values, k, v, cache_seqlens=state.seqlens,
                                              causal=True, window_size=window)
            new_state = state
        elif varlen is not None:
            out = ops.flash_attn_varlen_func(
                q.reshape(-1, self.num_heads, self.head_dim),
                k.reshape(-1, self.num_kv_heads, self.head_dim),
                v.reshape(-1, self.num_kv_heads, self.head_dim),
                cu_seqlens_q=varlen.cu_seqlens, cu_seqlens_k=varlen.cu_seqlens,
                max_seqlen_q=varlen.max_seqlen, max_seqlen_k=varlen.max_seqlen,
                causal=True, window_size=window)
        else:
            if state is not None:
                k = torch.cat([state.keys, k], dim=1)
                v = torch.cat([state.values, v], dim=1)
            if use_cache or self.shares_kv:
                keep = self.window if self.window is not None else self.max_seq_len
                new_state = KVCache(k[:, -keep:], v[:, -keep:])
            out = ops.flash_attn_func(q, k, v, causal=True, window_size=window)
        out = out.reshape(bsz, seq, -1)
        if self.gate_proj is not None:
            out = ops.sigmoid_gate(out, ops.linear(x, self.gate_proj.weight))
        return ops.linear(out, self.o_proj.weight), new_state


class SharedKV(nn.Module):
    """YOCO shared keys/values projected from the self-decoder output."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        a = config.attention
        self.num_kv_heads, self.head_dim = a.num_kv_heads, a.head_dim
        self.norm = RMSNorm(config.hidden_size, config.norm_eps)
        self.kv_proj = nn.Linear(config.hidden_size, 2 * a.num_kv_heads * a.head_dim, bias=False)
        self.k_norm = RMSNorm(a.head_dim, config.norm_eps) if a.qk_norm else None
        self.rope = RotaryEmbedding(a.head_dim, config.max_seq_len, a.rope_theta_global) if config.cross_rope else None

    def forward(self, x, position_ids, state: KVCache | None = None) -> KVCache:
        bsz, seq, _ = x.shape
        kv = ops.linear(self.norm(x, out_dtype=ops.compute_dtype(x)), self.kv_proj.weight)
        k, v = kv.view(bsz, seq, 2 * self.num_kv_heads, self.head_dim).chunk(2, dim=2)
        if self.k_norm is not None:
            k = self.k_norm(k, out_dtype=v.dtype)
        if self.rope is not None:
            k = self.rope.rotate(k, position_ids)
        if isinstance(state, StaticKV):
            bsz_, new = k.shape[:2]
            rows = torch.arange(bsz_, device=k.device)[:, None]
            cols = state.seqlens.long()[:, None] + torch.arange(new, device=k.device)
            state.keys[rows, cols] = k
            state.values[rows, cols] = v
            return state
        if state is not None:
            k = torch.cat([state.keys, k], dim=1)
            v = torch.cat([state.values, v], dim=1)
        return KVCache(k, v)


class CrossAttention(nn.Module):
    """YOCO cross-decoder attention over the shared KV (queries end-aligned to keys)."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        a = config.attention
        self.num_heads, self.num_kv_heads, self.head_dim = a.num_heads, a.num_kv_heads, a.head_dim
        qs = a.num_heads * a.head_dim
        self.q_proj = nn.Linear(config.hidden_size, qs, bias=False)
        self.o_proj = nn.Linear(qs, config.hidden_size, bias=False)
        self.q_norm = RMSNorm(a.head_dim, config.norm_eps) if a.qk_norm else None
        self.gate_proj = nn.Linear(config.hidden_size, qs, bias=False) if a.output_gate else None
        self.rope = RotaryEmbedding(a.head_dim, config.max_seq_len, a.rope_theta_global) if config.cross_rope else None

    def residual_projections(self) -> list[nn.Linear]:
        return [self.o_proj]

    def forward(self, x, position_ids, varlen: Varlen | None = None, state: KVCache | None = None,
                use_cache: bool = False):
        if state is None:
            raise ValueError("a cross-decoder block needs the shared KV as its state")
        bsz, seq, _ = x.shape
        q = ops.linear(x, self.q_proj.weight).view(bsz, seq, self.num_heads, self.head_dim)
        if self.q_norm is not None:
            q = self.q_norm(q, out_dtype=q.dtype)
        if self.rope is not None:
            q = self.rope.rotate(q, position_ids)
        out = self.attend(q, state, varlen).reshape(bsz, seq, -1)
        if self.gate_proj is not None:
            out = ops.sigmoid_gate(out, ops.linear(x, self.gate_proj.weight))
        return ops.linear(out, self.o_proj.weight), None

    def attend(self, q, kv, varlen: Varlen | None):
        if isinstance(kv, StaticKV):
            return ops.flash_attn_with_kvcache(q, kv.keys, kv.values, cache_seqlens=kv.seqlens + q.shape[1],
                                               causal=True)
        if varlen is None:
            return ops.flash_attn_func(q, kv.keys, kv.values, causal=True)
        return ops.flash_attn_varlen_func(
            q.reshape(-1, self.num_heads, self.head_dim),
            kv.keys.reshape(-1, self.num_kv_heads, self.head_dim),
            kv.values.reshape(-1, self.num_kv_heads, self.head_dim),
            cu_seqlens_q=varlen.cu_seqlens, cu_seqlens_k=varlen.cu_seqlens,
            max_seqlen_q=varlen.max_seqlen, max_seqlen_k=varlen.max_seqlen, causal=True)


# ---------------------------------------------------------------------------------------
# DeltaNet
# ---------------------------------------------------------------------------------------
class ShortConvolution(nn.Conv1d):
    """Depthwise causal convolution (weight (D, 1, K)); the parameter layout is
    ``torch.nn.Conv1d``'s so checkpoints match flash-linear-attention's module."""

    def __init__(self, hidden_size: int, kernel_size: int, bias: bool = False) -> None:
        super().__init__(hidden_size, hidden_size, kernel_size, groups=hidden_size, padding=kernel_size - 1, bias=bias)
        self.hidden_size = hidden_size


class GatedRMSNorm(nn.Module):
    """RMSNorm over the head dimension times swish(gate) (GDN) or sigmoid(gate) (KDA)."""

    def __init__(self, dim: int, eps: float = 1e-5, activation: str = "swish") -> None:
        super().__init__()
        self.eps, self.activation = eps, activation
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, o: torch.Tensor, gate: torch.Tensor | None = None) -> torch.Tensor:
        return ops.gated_rms_norm(o, gate, self.weight, self.eps, self.activation)


class DeltaNetInner(nn.Module):
    """Parameters of a Gated DeltaNet (``kind='gdn'``) or Kimi Delta Attention layer.

    Names, shapes and initialisation follow flash-linear-attention's layers (which the
    reference instantiates): q/k/v projections, ``a_proj`` (GDN) or the low-rank
    ``f_proj`` (KDA) for the decay, ``b_proj`` for beta, per-channel short convolutions,
    ``A_log`` / ``dt_bias`` for the decay gate, output gate ``g_proj`` and gated
    ``o_norm`` (eps 1e-5).
    """

    def __init__(self, hidden_size: int, kind: str, num_heads: int, head_dim: int, expand_v: float,
                 use_short_conv: bool, conv_size: int, use_gate: bool) -> None:
        super().__init__()
        self.kind = kind
        self.hidden_size = hidden_size
        self.num_heads = self.num_v_heads = num_heads
        self.head_k_dim = head_dim
        self.head_v_dim = int(head_dim * expand_v)
        self.key_dim = num_heads * head_dim
        self.value_dim = num_heads * self.head_v_dim
        self.use_short_conv, self.conv_size, self.conv_bias = use_short_conv, conv_size, False
        self.use_gate = use_gate or kind == "kda"
        self.allow_neg_eigval = False
        self.lower_bound = None
        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        if use_short_conv:
            self.q_conv1d = ShortConvolution(self.key_dim, conv_size)
            self.k_conv1d = ShortConvolution(self.key_dim, conv_size)
            self.v_conv1d = ShortConvolution(self.value_dim, conv_size)
        if kind == "kda":
            gate_dim = num_heads * head_dim
            self.f_proj = nn.Sequential(nn.Linear(hidden_size, self.head_v_dim, bias=False),
                                        nn.Linear(self.head_v_dim, gate_dim, bias=False))
            self.b_proj = nn.Linear(hidden_size, num_heads, bias=False)
            self.A_log = nn.Parameter(torch.log(torch.empty(num_heads).uniform_(1, 16)))
            self.dt_bias = nn.Parameter(self._inverse_softplus_dt(gate_dim))
            self.g_proj = nn.Sequential(nn.Linear(hidden_size, self.head_v_dim, bias=False),
                                        nn.Linear(self.head_v_dim, self.value_dim, bias=True))
            self.o_norm = GatedRMSNorm(self.head_v_dim, 1e-5, activation="sigmoid")
        else:
            self.a_proj = nn.Linear(hidden_size, num_heads, bias=False)
            self.b_proj = nn.Linear(hidden_size, num_heads, bias=False)
            self.A_log = nn.Parameter(torch.log(torch.empty(num_heads).uniform_(0, 16)))
            self.dt_bias = nn.Parameter(self._inverse_softplus_dt(num_heads))
            if use_gate:
                self.g_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
            self.o_norm = GatedRMSNorm(self.head_v_dim, 1e-5, activation="swish")
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)
        self.A_log._no_weight_decay = True
        self.dt_bias._no_weight_decay = True

    @staticmethod
    def _inverse_softplus_dt(n: int) -> torch.Tensor:
        lo, hi = math.log(1e-3), math.log(1e-1)
        dt = torch.exp(torch.rand(n) * (hi - lo) + lo).clamp(min=1e-4)
        return dt + torch.log(-torch.expm1(-dt))

    def conv_weight(self) -> torch.Tensor:
        """(2*key_dim + value_dim, K) stacked q/k/v convolution weights."""
        return torch.cat([self.q_conv1d.weight, self.k_conv1d.weight, self.v_conv1d.weight], 0).squeeze(1)


@dataclass
class DeltaState:
    """Decode cache of a DeltaNet layer: last K-1 conv inputs and the recurrent state."""

    conv: torch.Tensor | None  # (batch, 2*key_dim+value_dim, K-1)
    recurrent: torch.Tensor  # (batch, heads, head_k_dim, head_v_dim) fp32


class SpecDeltaState:
    """Static decode cache of a DeltaNet layer for speculative decoding.

    Holds the committed conv inputs (batch, channels, K-1) and recurrent state (batch,
    heads, dk, dv) fp32, plus the previous window's inputs, of which row b accepted the
    first ``pending[b]`` tokens (``pending`` int32 is shared by all layers and set by the
    decoder after verification).  A window call commits that accepted prefix first, then
    runs the new window without committing it, so rejected drafts never reach the state.
    ``prefill`` switches a call to a plain pass from the committed state (which it then
    replaces); the decoder sets it around the prompt pass.  All buffers are static, so a
    round can be captured in a CUDA graph.
    """

    def __init__(self, inner: "DeltaNetInner", batch: int, window: int, pending: torch.Tensor,
                 dtype: torch.dtype, device: torch.device) -> None:
        h, dk, dv = inner.num_heads, inner.head_k_dim, inner.head_v_dim
        channels = 2 * inner.key_dim + inner.value_dim
        self.window, self.pending, self.prefill = window, pending, False
        self.conv = (torch.zeros(batch, channels, inner.conv_size - 1, dtype=dtype, device=device)
                     if inner.use_short_conv else None)
        self.window_x = torch.zeros(batch, window, channels, dtype=dtype, device=device) if inner.use_short_conv else None
        self.recurrent = torch.zeros(batch, h, dk, dv, dtype=torch.float32, device=device)
        gdim = (h, dk) if inner.kind == "kda" else (h,)
        self.inputs = (torch.zeros(batch, window, h, dk, dtype=dtype, device=device),
                       torch.zeros(batch, window, h, dk, dtype=dtype, device=device),
                       torch.zeros(batch, window, h, dv, dtype=dtype, device=device),
                       torch.zeros(batch, window, *gdim, dtype=torch.float32, device=device),
                       torch.zeros(batch, window, h, dtype=torch.float32, device=device))

    def reset(self) -> None:
        self.recurrent.zero_()
        if self.conv is not None:
            self.conv.zero_()

    def commit_conv(self, raw: torch.Tensor) -> None:
        """Conv inputs: fold the accepted prefix of the last window into the committed
        state, then keep this window's raw inputs ``raw`` (batch, W, channels)."""
        if self.conv is None:
            return
        span = torch.cat([self.conv, self.window_x.transpose(1, 2)], 2)  # (B, C, K-1+W)
        idx = self.pending.long()[:, None] + torch.arange(self.conv.size(2), device=span.device)[None]
        self.conv.copy_(span.gather(2, idx[:, None, :].expand(-1, span.size(1), -1)))
        self.window_x.copy_(raw)


class DeltaNet(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        c = config.deltanet
        self.kind = c.kind
        self.inner = DeltaNetInner(config.hidden_size, c.kind, c.num_heads, c.head_dim, c.expand_v,
                                   c.use_short_conv, c.conv_size, c.use_gate)

    def residual_projections(self) -> list[nn.Linear]:
        return [self.inner.o_proj]

    def forward(self, x, position_ids, varlen: Varlen | None = None, state: DeltaState | None = None,
                use_cache: bool = False):
        inner = self.inner
        bsz, seq, hidden = x.shape
        packed = varlen is not None
        h = x.reshape(1, bsz * seq, hidden) if packed else x
        cu = varlen.cu_seqlens if packed else None
        cu_cpu = varlen.cu_seqlens_cpu if packed else None
        qkv = torch.cat([ops.linear(h, inner.q_proj.weight), ops.linear(h, inner.k_proj.weight),
                         ops.linear(h, inner.v_proj.weight)], dim=-1)
        if self.kind == "kda":
            f = ops.linear(ops.linear(h, inner.f_proj[0].weight), inner.f_proj[1].weight)
            raw_gate = f
        else:
            raw_gate = ops.linear(h, inner.a_proj.weight)
        b = ops.linear(h, inner.b_proj.weight)
        if inner.use_gate:
            if self.kind == "kda":
                og = ops.linear(ops.linear(h, inner.g_proj[0].weight), inner.g_proj[1].weight) + inner.g_proj[1].bias
            else:
                og = ops.linear(h, inner.g_proj.weight)
        else:
            og = None
        spec = isinstance(state, SpecDeltaState)
        if spec and not state.prefill:
            return self._spec_window(qkv, raw_gate, b, og, state), state
        conv_state = state.conv if state is not None else None
        if inner.use_short_conv:
            qkv, new_conv = ops.causal_conv1d(qkv, inner.conv_weight(), cu_seqlens=cu, initial_state=conv_state,
                                              return_final_state=use_cache)
        else:
            qkv, new_conv = ops.silu(qkv), None
        b_, t_ = qkv.shape[:2]
        q, k, v = ops.split_cols(qkv, (inner.key_dim, inner.key_dim, inner.value_dim))
        q = q.reshape(b_, t_, inner.num_heads, inner.head_k_dim)
        k = k.reshape(b_, t_, inner.num_heads, inner.head_k_dim)
        v = v.reshape(b_, t_, inner.num_v_heads, inner.head_v_dim)
        if self.kind == "kda":
            g = ops.kda_gate(raw_gate.reshape(b_, t_, inner.num_heads, inner.head_k_dim), inner.A_log, inner.dt_bias)
        else:
            g = ops.gdn_gate(raw_gate, inner.A_log, inner.dt_bias)
        beta = torch.sigmoid(b.float())
        init = state.recurrent if state is not None else None
        o, final = ops.gated_delta_rule(q, k, v, g, beta, initial_state=init, cu_seqlens=cu,
                                        cu_seqlens_cpu=cu_cpu, output_final_state=use_cache,
                                        per_channel_decay=self.kind == "kda")
        o = inner.o_norm(o, og.reshape(b_, t_, inner.num_v_heads, inner.head_v_dim) if og is not None else None)
        out = ops.linear(o.reshape(b_, t_, inner.value_dim), inner.o_proj.weight)
        if packed:
            out = out.reshape(bsz, seq, hidden)
        if spec:  # prefill of a speculative decoder: the prompt's final states become committed
            if new_conv is not None:
                state.conv.copy_(new_conv)
            state.recurrent.copy_(final)
            return out, state
        new_state = DeltaState(new_conv, final) if use_cache else None
        return out, new_state

    def _spec_window(self, qkv, raw_gate, b, og, state: SpecDeltaState):
        """One speculative window (batch layout, W = state.window tokens)."""
        inner = self.inner
        b_, t_ = qkv.shape[:2]
        if t_ != state.window:
            raise ValueError(f"speculative window of {t_} tokens, the cache was built for {state.window}")
        if inner.use_short_conv:
            state.commit_conv(qkv)
            qkv, _ = ops.causal_conv1d(qkv, inner.conv_weight(), initial_state=state.conv)
        else:
            qkv = ops.silu(qkv)
        q, k, v = ops.split_cols(qkv, (inner.key_dim, inner.key_dim, inner.value_dim))
        q = q.reshape(b_, t_, inner.num_heads, inner.head_k_dim)
        k = k.reshape(b_, t_, inner.num_heads, inner.head_k_dim)
        v = v.reshape(b_, t_, inner.num_v_heads, inner.head_v_dim)
        if self.kind == "kda":
            g = ops.kda_gate(raw_gate.reshape(b_, t_, inner.num_heads, inner.head_k_dim), inner.A_log, inner.dt_bias)
        else:
            g = ops.gdn_gate(raw_gate, inner.A_log, inner.dt_bias)
        beta = torch.sigmoid(b.float())
        o = ops.delta_spec_window(q, k, v, g, beta, state.recurrent, state.inputs, state.pending,
                                  per_channel_decay=self.kind == "kda")
        o = inner.o_norm(o, og.reshape(b_, t_, inner.num_v_heads, inner.head_v_dim) if og is not None else None)
        return ops.linear(o.reshape(b_, t_, inner.value_dim), inner.o_proj.weight)


def build_mixer(config: ModelConfig, layer_type: str, first_global: bool) -> nn.Module:
    if layer_type == LOCAL_ATTENTION:
        return Attention(config, local=True, use_rope=True)
    if layer_type == GLOBAL_ATTENTION:
        mode = config.attention.global_rope
        return Attention(config, local=False, use_rope=mode == "all" or (mode == "first" and first_global))
    if layer_type == DELTANET:
        return DeltaNet(config)
    if layer_type == CROSS_ATTENTION:
        return CrossAttention(config)
    raise ValueError(f"unknown layer type {layer_type!r}")
