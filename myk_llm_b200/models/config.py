"""Model hyper-parameters.

Field names, defaults and validation rules follow the upstream schema
(reference: ``src/myk_llm/model/config.py:17-263``) so a ``model:`` section written for
the reference describes the same network here, and ``model.yaml`` files exported by
either side load in the other.

Layer codes (one character per block, the pattern repeats to ``num_layers``):

* ``G`` global causal softmax attention
* ``L`` sliding-window causal softmax attention
* ``D`` Gated DeltaNet (or Kimi Delta Attention) linear attention
* ``X`` cross-decoder block of a decoder-decoder (YOCO) model
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal

GLOBAL_ATTENTION = "G"
LOCAL_ATTENTION = "L"
DELTANET = "D"
CROSS_ATTENTION = "X"
LAYER_CODES = (GLOBAL_ATTENTION, LOCAL_ATTENTION, DELTANET, CROSS_ATTENTION)


@dataclass
class AttentionConfig:
    num_heads: int = 8
    num_kv_heads: int = 2
    head_dim: int = 128
    sliding_window: int = 512
    rope_theta_local: float = 10_000.0
    rope_theta_global: float = 1_000_000.0
    # Which "G" layers rotate q/k: only the first global layer, all of them, or none
    # (NoPE).  "L" layers always rotate.
    global_rope: Literal["first", "all", "none"] = "first"
    qk_norm: bool = False
    output_gate: bool = False


@dataclass
class DeltaNetConfig:
    kind: Literal["gdn", "kda"] = "gdn"
    num_heads: int = 8
    head_dim: int = 128
    expand_v: float = 1.0
    conv_size: int = 4
    use_short_conv: bool = True
    use_gate: bool = True


@dataclass
class FFNConfig:
    multiplier: float = 4.0
    multiple_of: int = 256


@dataclass
class ResidualConfig:
    """x + gate * f(norm(x)); gate is 1 (none), a learned scalar, a learned vector, or
    2*sigmoid(W norm(x)) with W initialised to zero (input)."""

    gate: Literal["none", "scalar", "channel", "input"] = "none"
    init: float = 1.0


@dataclass
class NgramEmbeddingConfig:
    """Hashed n-gram input embeddings (one table per order, summed), injected into the
    inputs of the blocks listed in ``layers`` through one projection each."""

    orders: list[int] = field(default_factory=list)
    num_buckets: int = 131_072
    dim: int = 256
    layers: list[int] = field(default_factory=lambda: [0])


@dataclass
class MTPConfig:
    """DeepSeek-V3 style multi-token prediction: ``depth`` chained modules, module k
    predicts token t+1+k."""

    depth: int = 0
    layer: str = GLOBAL_ATTENTION


@dataclass
class LoopConfig:
    """Looped core: blocks [prelude, prelude+core) share weights over ``iterations``
    passes; training may draw the count from ``train_iterations`` and backpropagate
    through only the last ``backprop_iterations``."""

    core: int = 0
    prelude: int = 0
    iterations: int = 1
    train_iterations: list[int] = field(default_factory=list)
    backprop_iterations: int = 0
    injection: Literal["add", "concat"] = "add"


@dataclass
class CrossDecoderConfig:
    """Decoder-decoder: the shared KV is projected from the self-decoder output
    (``project``) or taken from the self-decoder's last global layer (``layer``)."""

    kv: Literal["project", "layer"] = "project"


@dataclass
class ModelConfig:
    vocab_size: int = 65536
    hidden_size: int = 1024
    num_layers: int = 9
    layer_pattern: str = "GL"
    max_seq_len: int = 4096
    parallel_block: bool = False
    parallel_streams: bool = False
    norm_eps: float = 1e-6
    tie_embeddings: bool = True
    initializer_range: float = 0.02
    attention: AttentionConfig = field(default_factory=AttentionConfig)
    deltanet: DeltaNetConfig = field(default_factory=DeltaNetConfig)
    ffn: FFNConfig = field(default_factory=FFNConfig)
    residual: ResidualConfig = field(default_factory=ResidualConfig)
    ngram: NgramEmbeddingConfig = field(default_factory=NgramEmbeddingConfig)
    mtp: MTPConfig = field(default_factory=MTPConfig)
    loop: LoopConfig = field(default_factory=LoopConfig)
    cross: CrossDecoderConfig = field(default_factory=CrossDecoderConfig)

    def __post_init__(self) -> None:
        self._validate()

    # -- validation --------------------------------------------------------------------
    def _validate(self) -> None:
        pattern = self.layer_pattern
        if not pattern or any(c not in LAYER_CODES for c in pattern):
            raise ValueError(f"layer_pattern must use only {LAYER_CODES}, got {pattern!r}")
        att = self.attention
        if att.num_heads % att.num_kv_heads:
            raise ValueError("attention.num_heads must be divisible by attention.num_kv_heads")
        ng = self.ngram
        if any(o < 2 for o in ng.orders):
            raise ValueError("ngram.orders must be >= 2 (order 1 is the token embedding)")
        if ng.orders:
            ok = bool(ng.layers) and len(set(ng.layers)) == len(ng.layers)
            ok = ok and all(0 <= i < self.num_layers for i in ng.layers)
            if not ok:
                raise ValueError(f"ngram.layers must be distinct block indices in [0, {self.num_layers}), got {ng.layers}")
        if self.mtp.layer not in (GLOBAL_ATTENTION, LOCAL_ATTENTION, DELTANET):
            raise ValueError(f"mtp.layer must be one of {LAYER_CODES[:-1]}")
        kinds, xs = self.layer_types, self.cross_start
        loop = self.loop
        if xs < self.num_layers:
            tail_ok = set(kinds[xs:]) == {CROSS_ATTENTION} and CROSS_ATTENTION not in kinds[:xs]
            if xs == 0 or not tail_ok:
                raise ValueError(
                    "cross-decoder ('X') blocks must be the last blocks after at least one other, "
                    f"got {''.join(kinds)} (write the pattern out in full, e.g. LLLLXXXX)")
            if loop.core and loop.prelude < xs < loop.prelude + loop.core:
                raise ValueError(
                    f"the loop core (blocks {loop.prelude}-{loop.prelude + loop.core - 1}) must lie "
                    f"either before the cross-decoder or inside it (from block {xs})")
            if self.cross.kv == "layer" and GLOBAL_ATTENTION not in kinds[:xs]:
                raise ValueError("cross.kv=layer needs a global ('G') layer in the self-decoder")
        if loop.core < 0 or loop.prelude < 0 or loop.prelude + loop.core > self.num_layers:
            raise ValueError(f"need loop.core, loop.prelude >= 0 and prelude + core <= num_layers ({self.num_layers})")
        if loop.core:
            if loop.iterations < 1 or loop.backprop_iterations < 0:
                raise ValueError("need loop.iterations >= 1 and loop.backprop_iterations >= 0")
            ti = loop.train_iterations
            if ti and (len(ti) != 2 or not 1 <= ti[0] <= ti[1]):
                raise ValueError(f"loop.train_iterations must be [min, max] with 1 <= min <= max, got {ti}")
            inside = range(loop.prelude + 1, loop.prelude + loop.core)
            if ng.orders and any(i in inside for i in ng.layers):
                raise ValueError("ngram.layers cannot point inside the loop core (except at its first block)")

    # -- derived properties ------------------------------------------------------------
    @property
    def layer_types(self) -> list[str]:
        p = self.layer_pattern
        return [p[i % len(p)] for i in range(self.num_layers)]

    @property
    def cross_start(self) -> int:
        kinds = self.layer_types
        return kinds.index(CROSS_ATTENTION) if CROSS_ATTENTION in kinds else self.num_layers

    @property
    def cross_kv_layer(self) -> int | None:
        xs = self.cross_start
        if xs == self.num_layers or self.cross.kv != "layer":
            return None
        return max(i for i, t in enumerate(self.layer_types[:xs]) if t == GLOBAL_ATTENTION)

    @property
    def cross_rope(self) -> bool:
        mode = self.attention.global_rope
        globals_ = [i for i, t in enumerate(self.layer_types) if t == GLOBAL_ATTENTION]
        src = self.cross_kv_layer
        is_first = (src == globals_[0]) if src is not None else not globals_
        return mode == "all" or (mode == "first" and is_first)

    @property
    def effective_layers(self) -> int:
        return self.num_layers + self.loop.core * (self.loop.iterations - 1)

    @property
    def layout(self) -> str:
        kinds, loop = "".join(self.layer_types), self.loop
        if not loop.core:
            return kinds
        end = loop.prelude + loop.core
        return f"{kinds[:loop.prelude]}({kinds[loop.prelude:end]})x{loop.iterations}{kinds[end:]}"

    @property
    def ffn_hidden_size(self) -> int:
        raw = int(self.hidden_size * self.ffn.multiplier)
        m = self.ffn.multiple_of
        return m * ((raw + m - 1) // m)
