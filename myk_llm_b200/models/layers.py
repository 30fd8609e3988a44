"""Building blocks shared by mixers and blocks.

Parameter names and shapes match the upstream modules (reference:
``src/myk_llm/model/layers.py:15-115``), because they are part of the checkpoint
contract.  The arithmetic goes through :mod:`myk_llm_b200.ops`, which runs the sm_100a
kernels on CUDA tensors and the PyTorch statements on CPU tensors.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import ops
from .config import ModelConfig, ResidualConfig


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight, weight kept in fp32."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps, out_dtype=out_dtype)


class SwiGLU(nn.Module):
    """down(silu(gate) * up) with one fused ``up_gate_proj`` whose rows [0, F) are the gate
    and rows [F, 2F) the up projection."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        f = config.ffn_hidden_size
        self.up_gate_proj = nn.Linear(config.hidden_size, 2 * f, bias=False)
        self.down_proj = nn.Linear(f, config.hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gu = ops.linear(x, self.up_gate_proj.weight)
        return ops.linear(ops.swiglu(gu), self.down_proj.weight)


class ResidualGate(nn.Module):
    """How a sublayer update joins the residual stream (see ResidualConfig)."""

    def __init__(self, config: ResidualConfig, hidden_size: int) -> None:
        super().__init__()
        self.kind = config.gate
        if self.kind == "scalar":
            self.scale = nn.Parameter(torch.full((1,), config.init))
        elif self.kind == "channel":
            self.scale = nn.Parameter(torch.full((hidden_size,), config.init))
        elif self.kind == "input":
            self.gate_proj = nn.Linear(hidden_size, hidden_size, bias=False)

    def init_weights(self) -> None:
        if self.kind == "input":
            nn.init.zeros_(self.gate_proj.weight)

    def scaled(self, update: torch.Tensor, normed_input: torch.Tensor) -> torch.Tensor:
        """gate * update (the part added to the residual)."""
        if self.kind == "none":
            return update
        if self.kind == "input":
            g = ops.linear(normed_input, self.gate_proj.weight)
            return 2.0 * torch.sigmoid(g.float()) * update
        return self.scale * update

    def forward(self, residual: torch.Tensor, update: torch.Tensor, normed_input: torch.Tensor) -> torch.Tensor:
        return residual + self.scaled(update, normed_input)


class RotaryEmbedding(nn.Module):
    """RoPE with interleaved pairs (dims 2i and 2i+1 rotate together), fp32 tables.

    The cos/sin tables are non-persistent buffers that stay fp32 when the module is cast.
    """

    def __init__(self, head_dim: int, max_seq_len: int, base: float) -> None:
        super().__init__()
        if head_dim % 2:
            raise ValueError("head_dim must be even for RoPE")
        self.head_dim, self.base = head_dim, base
        self._build(max_seq_len)

    def _build(self, length: int, device: torch.device | None = None) -> None:
        half = torch.arange(0, self.head_dim, 2, dtype=torch.float32, device=device) / self.head_dim
        inv_freq = 1.0 / (self.base ** half)
        pos = torch.arange(length, dtype=torch.float32, device=device)
        ang = torch.outer(pos, inv_freq).repeat_interleave(2, dim=-1)
        self.register_buffer("cos_cached", ang.cos(), persistent=False)
        self.register_buffer("sin_cached", ang.sin(), persistent=False)

    def _apply(self, fn, recurse: bool = True):
        super()._apply(fn, recurse=recurse)
        self.cos_cached = self.cos_cached.float()
        self.sin_cached = self.sin_cached.float()
        return self

    def rotate(self, x: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
        """Rotate (batch, seq, heads, head_dim) to ``position_ids`` (batch, seq)."""
        return ops.apply_rope(x, self.cos_cached, self.sin_cached, position_ids)

    def forward(self, q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor):
        return self.rotate(q, position_ids), self.rotate(k, position_ids)

    def split_qkv(self, qkv: torch.Tensor, position_ids: torch.Tensor, heads: int, kv_heads: int):
        """Rotated q, k and v from a fused QKV projection (one pass over it)."""
        return ops.rope_qkv(qkv, self.cos_cached, self.sin_cached, position_ids, heads, kv_heads)


def init_linear_(module: nn.Module, std: float) -> None:
    if isinstance(module, (nn.Linear, nn.Embedding)):
        nn.init.normal_(module.weight, mean=0.0, std=std)
        if getattr(module, "bias", None) is not None:
            nn.init.zeros_(module.bias)


def residual_init_scale(num_layers: int) -> float:
    return 1.0 / math.sqrt(2 * num_layers)
