"""Ops layer: every hot op of the model, trainer and decoder.

CUDA tensors run the hand-written sm_100a kernels of ``myk_llm_b200._C`` (built from
``csrc/``); CPU tensors run the PyTorch statements in :mod:`.reference`, which are also
the fp32 oracles of the kernel tests.  There is no other backend.
"""

from ._ext import available, compute_dtype, ext, is_cuda
from .attention import flash_attn_func, flash_attn_varlen_func, flash_attn_with_kvcache
from .elementwise import (add_rms_norm, apply_rope, rope_qkv, embedding, gated_rms_norm, ngram_lookup, rms_norm,
                          sigmoid_gate, silu, split_cols, swiglu)
from .gdn import causal_conv1d, gated_delta_rule, gdn_gate, kda_gate
from .gdn import spec_window as delta_spec_window
from .linear import bf16_weight, gemm, invalidate_weight_cache, linear
from .loss import fused_linear_cross_entropy
from .optim_kernels import (adamw_multi_tensor, batched_newton_schulz_orthogonalize, batched_syrk,
                            frobenius_normalize_, muon_apply, muon_prepare)

__all__ = [
    "adamw_multi_tensor", "add_rms_norm", "apply_rope", "available", "batched_newton_schulz_orthogonalize",
    "batched_syrk", "bf16_weight", "causal_conv1d", "compute_dtype", "delta_spec_window", "embedding", "ext", "flash_attn_func",
    "flash_attn_varlen_func", "flash_attn_with_kvcache", "frobenius_normalize_", "fused_linear_cross_entropy",
    "gated_delta_rule", "gated_rms_norm", "gdn_gate", "gemm", "invalidate_weight_cache", "is_cuda", "kda_gate", "linear", "muon_apply",
    "muon_prepare", "ngram_lookup", "rms_norm", "rope_qkv", "sigmoid_gate", "silu", "split_cols", "swiglu",
]
