"""Model hyper-parameters.

Field names and defaults are the reference's schema (``src/myk_llm/model/config.py:17-175``)
so a ``model:`` section written for the reference describes the same network here, and
``model.yaml`` files exported by either side load in the other; the same configurations
are rejected (the rules are the table ``_RULES`` at the end of this file), and the
derived layout properties keep the reference's names and meaning.

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
        for rule in _RULES:
            problem = rule(self)
            if problem:
                raise ValueError(problem)

    # -- derived layout (the names are the reference's public properties) ---------------
    @property
    def layer_types(self) -> list[str]:
        """One layer code per block: the pattern repeated to ``num_layers``."""
        reps = -(-self.num_layers // len(self.layer_pattern))
        return list((self.layer_pattern * reps)[:self.num_layers])

    @property
    def cross_start(self) -> int:
        """Index of the first cross-decoder block (``num_layers`` when there is none)."""
        return "".join(self.layer_types).find(CROSS_ATTENTION) % (self.num_layers + 1)

    @property
    def cross_kv_layer(self) -> int | None:
        """The self-decoder block whose keys / values the cross-decoder reuses
        (``cross.kv == "layer"``): the last global block before the cross-decoder."""
        start = self.cross_start
        if start == self.num_layers or self.cross.kv != "layer":
            return None
        return "".join(self.layer_types[:start]).rfind(GLOBAL_ATTENTION)

    def rotates(self, block: int) -> bool:
        """Whether the attention of a G / L block applies RoPE: local blocks always; global
        blocks by ``attention.global_rope`` (all, only the first global block, or none)."""
        kind = self.layer_types[block]
        if kind == LOCAL_ATTENTION:
            return True
        mode = self.attention.global_rope
        return mode == "all" or (mode == "first" and block == "".join(self.layer_types).find(GLOBAL_ATTENTION))

    @property
    def cross_rope(self) -> bool:
        """Whether the shared keys (and so the cross-decoder queries) are rotated: as the
        source block when the KV comes from a layer, else as a first global block would be
        (rotated under "first" only when the model has no global block at all)."""
        src = self.cross_kv_layer
        if src is not None:
            return self.rotates(src)
        mode = self.attention.global_rope
        return mode == "all" or (mode == "first" and GLOBAL_ATTENTION not in self.layer_types)

    @property
    def effective_layers(self) -> int:
        """Blocks run per forward pass at the default iteration count."""
        return self.num_layers + self.loop.core * (self.loop.iterations - 1)

    @property
    def layout(self) -> str:
        """Layer codes with the looped core marked, e.g. ``D(GD)x4G``."""
        codes, lp = "".join(self.layer_types), self.loop
        if not lp.core:
            return codes
        a, b = lp.prelude, lp.prelude + lp.core
        return f"{codes[:a]}({codes[a:b]})x{lp.iterations}{codes[b:]}"

    @property
    def ffn_hidden_size(self) -> int:
        """``hidden_size * ffn.multiplier`` rounded up to a multiple of ``ffn.multiple_of``."""
        raw, unit = int(self.hidden_size * self.ffn.multiplier), self.ffn.multiple_of
        return -(-raw // unit) * unit


# -- validation rules: each returns an error message or None ----------------------------
def _rule_pattern(c: ModelConfig):
    if not c.layer_pattern or not set(c.layer_pattern) <= set(LAYER_CODES):
        return f"layer_pattern must use only {LAYER_CODES}, got {c.layer_pattern!r}"


def _rule_heads(c: ModelConfig):
    if c.attention.num_heads % c.attention.num_kv_heads:
        return "attention.num_heads must be divisible by attention.num_kv_heads"


def _rule_ngram(c: ModelConfig):
    ng = c.ngram
    if min(ng.orders, default=2) < 2:
        return "ngram.orders must be >= 2 (order 1 is the token embedding)"
    if ng.orders and not (ng.layers and len(set(ng.layers)) == len(ng.layers)
                          and all(0 <= i < c.num_layers for i in ng.layers)):
        return f"ngram.layers must be distinct block indices in [0, {c.num_layers}), got {ng.layers}"


def _rule_mtp(c: ModelConfig):
    if c.mtp.layer not in (GLOBAL_ATTENTION, LOCAL_ATTENTION, DELTANET):
        return f"mtp.layer must be one of {LAYER_CODES[:-1]}"


def _rule_loop_bounds(c: ModelConfig):
    lp = c.loop
    if min(lp.core, lp.prelude) < 0 or lp.prelude + lp.core > c.num_layers:
        return f"need loop.core, loop.prelude >= 0 and prelude + core <= num_layers ({c.num_layers})"
    if not lp.core:
        return None
    if lp.iterations < 1 or lp.backprop_iterations < 0:
        return "need loop.iterations >= 1 and loop.backprop_iterations >= 0"
    ti = lp.train_iterations
    if ti and not (len(ti) == 2 and 1 <= ti[0] <= ti[1]):
        return f"loop.train_iterations must be [min, max] with 1 <= min <= max, got {ti}"
    # a core block after the first runs on the loop state, which has no single input to
    # inject into; the first core block's injection joins the loop input
    if c.ngram.orders and any(lp.prelude < i < lp.prelude + lp.core for i in c.ngram.layers):
        return "ngram.layers cannot point inside the loop core (except at its first block)"


def _rule_cross(c: ModelConfig):
    codes = "".join(c.layer_types)
    start = c.cross_start
    if start == c.num_layers:
        return None
    if start == 0 or codes[start:].strip(CROSS_ATTENTION):
        return ("cross-decoder ('X') blocks must be the last blocks after at least one other, "
                f"got {codes} (write the pattern out in full, e.g. LLLLXXXX)")
    lp = c.loop
    if lp.core and lp.prelude < start < lp.prelude + lp.core:
        return (f"the loop core (blocks {lp.prelude}-{lp.prelude + lp.core - 1}) must lie either before the "
                f"cross-decoder or inside it (from block {start})")
    if c.cross.kv == "layer" and GLOBAL_ATTENTION not in codes[:start]:
        return "cross.kv=layer needs a global ('G') layer in the self-decoder"


_RULES = (_rule_pattern, _rule_heads, _rule_ngram, _rule_mtp, _rule_cross, _rule_loop_bounds)
