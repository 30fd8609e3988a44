"""Loader for the compiled sm_100a extension ``myk_llm_b200._C``.

CUDA tensors always take the kernel path.  If the extension is missing on a machine
with a GPU the op raises instead of silently falling back to PyTorch, so a test that
passes on CUDA has run the native code.
"""

from __future__ import annotations

import torch

_EXT = None
_ERR: Exception | None = None


def ext():
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        from .. import _C  # type: ignore[attr-defined]
    except ImportError as err:  # pragma: no cover - depends on the build
        _ERR = err
        raise RuntimeError(
            "myk_llm_b200._C (the sm_100a kernels) is not built; run `python setup.py build_ext --inplace` "
            "at the repository root") from err
    _EXT = _C
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def is_cuda(*tensors: torch.Tensor | None) -> bool:
    return any(t is not None and t.is_cuda for t in tensors)


def compute_dtype(x: torch.Tensor) -> torch.dtype:
    """Activation dtype of the compute path: bf16 on CUDA, the input dtype on CPU."""
    return torch.bfloat16 if x.is_cuda else x.dtype
