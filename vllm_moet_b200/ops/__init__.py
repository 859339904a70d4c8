"""Native op library (``vllm_moet_b200._C``, built from ``csrc/``).

On a machine with a GPU the extension is mandatory: :func:`native` raises
instead of silently falling back to PyTorch, so a missing build can never
masquerade as a working GPU run.  CPU-only runs (tests, the tiny CPU
config) use the pure-PyTorch reference ops in :mod:`.reference`.
"""
from __future__ import annotations

import importlib

import torch

_C = None
_err = None


def native():
    """Return the compiled extension module or raise a clear error."""
    global _C, _err
    if _C is not None:
        return _C
    try:
        mod = importlib.import_module("vllm_moet_b200._C")
        from .fingerprint import check_build
        check_build(mod)
        _C = mod
    except ImportError as e:  # pragma: no cover - depends on the build
        _err = e
        raise RuntimeError(
            "vllm_moet_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {e})") from e
    return _C


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


def require_gpu_native(device) -> None:
    if torch.device(device).type == "cuda":
        native()
