"""Building blocks shared by mixers and blocks: RMSNorm, SwiGLU, residual gates, RoPE and
the initialisation helpers.

Parameter names and shapes are part of the checkpoint contract with the reference
(``src/myk_llm/model/layers.py:15-115``); the arithmetic runs through
:mod:`myk_llm_b200.ops` (the sm_100a kernels for CUDA tensors, the PyTorch statements
for CPU tensors).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from .config import ModelConfig, ResidualConfig


class RMSNorm(nn.Module):
    """``x / rms(x) * weight`` with an fp32 weight; ``out_dtype`` lets the kernel write
    its result directly in the dtype the next GEMM reads."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps, out_dtype=out_dtype)


class SwiGLU(nn.Module):
    """``down(silu(g) * u)``; ``up_gate_proj`` stacks the gate rows [0, F) over the up rows
    [F, 2F), so one GEMM produces both and one kernel applies the activation."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        width = config.ffn_hidden_size
        self.up_gate_proj = nn.Linear(config.hidden_size, 2 * width, bias=False)
        self.down_proj = nn.Linear(width, config.hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(ops.swiglu(ops.linear(x, self.up_gate_proj.weight)), self.down_proj.weight)


class ResidualGate(nn.Module):
    """How a sublayer's update joins the residual stream: ``residual + g * update`` with
    ``g`` = 1 (``none``), a learned scalar (``scalar``), a learned vector (``channel``) or
    ``2 sigmoid(W norm(x))`` from the sublayer's normed input with ``W`` starting at zero
    (``input``, so every gate starts at 1)."""

    def __init__(self, config: ResidualConfig, hidden_size: int) -> None:
        super().__init__()
        self.kind = config.gate
        shapes = {"scalar": (1,), "channel": (hidden_size,)}
        if self.kind in shapes:
            self.scale = nn.Parameter(torch.full(shapes[self.kind], float(config.init)))
        elif self.kind == "input":
            self.gate_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        elif self.kind != "none":
            raise ValueError(f"unknown residual gate {self.kind!r}")

    def init_weights(self) -> None:
        if self.kind == "input":
            nn.init.zeros_(self.gate_proj.weight)

    def scaled(self, update: torch.Tensor, normed_input: torch.Tensor) -> torch.Tensor:
        """The part added to the residual stream."""
        if self.kind == "none":
            return update
        if self.kind == "input":
            return torch.sigmoid(ops.linear(normed_input, self.gate_proj.weight).float()).mul(2.0) * update
        return self.scale * update

    def forward(self, residual: torch.Tensor, update: torch.Tensor, normed_input: torch.Tensor) -> torch.Tensor:
        return residual + self.scaled(update, normed_input)


def rope_tables(head_dim: int, length: int, base: float, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 (length, head_dim) cos / sin tables with interleaved pairs: dims 2i and 2i+1
    rotate together at frequency ``1 / base ** (2i / head_dim)``.  The angles are formed
    in fp32 with the same operations as the reference's tables, so a model rotates by
    bit-identical angles in both frameworks."""
    exponent = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim
    freq = 1.0 / (base ** exponent)
    angle = torch.outer(torch.arange(length, dtype=torch.float32, device=device), freq)
    angle = angle.repeat_interleave(2, dim=1)
    return angle.cos(), angle.sin()


class RotaryEmbedding(nn.Module):
    """RoPE over fp32 tables of ``max_seq_len`` positions, kept fp32 when the module is cast
    (non-persistent buffers: not part of checkpoints)."""

    def __init__(self, head_dim: int, max_seq_len: int, base: float) -> None:
        super().__init__()
        if head_dim % 2:
            raise ValueError("head_dim must be even for RoPE")
        self.head_dim, self.base = head_dim, base
        cos, sin = rope_tables(head_dim, max_seq_len, base)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)

    def _apply(self, fn, recurse: bool = True):
        super()._apply(fn, recurse=recurse)
        self.cos_cached, self.sin_cached = self.cos_cached.float(), self.sin_cached.float()
        return self

    def rotate(self, x: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
        """(batch, seq, heads, head_dim) rotated to ``position_ids`` (batch, seq)."""
        return ops.apply_rope(x, self.cos_cached, self.sin_cached, position_ids)

    def forward(self, q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor):
        return self.rotate(q, position_ids), self.rotate(k, position_ids)

    def split_qkv(self, qkv: torch.Tensor, position_ids: torch.Tensor, heads: int, kv_heads: int):
        """Rotated q, k and v from a fused QKV projection in one pass (one kernel on CUDA)."""
        return ops.rope_qkv(qkv, self.cos_cached, self.sin_cached, position_ids, heads, kv_heads)


def init_linear_(module: nn.Module, std: float) -> None:
    """Normal(0, std) weights and zero biases for linears and embeddings."""
    if not isinstance(module, (nn.Linear, nn.Embedding)):
        return
    with torch.no_grad():
        module.weight.normal_(0.0, std)
        if getattr(module, "bias", None) is not None:
            module.bias.zero_()


def residual_init_scale(num_layers: int) -> float:
    """Output projections start scaled by 1/sqrt(2 L) (two residual updates per block)."""
    return (2.0 * num_layers) ** -0.5
