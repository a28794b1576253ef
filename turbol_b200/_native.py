"""Loader for the native core (``turbol_b200/turbol_core*.so``).

The extension is built in-tree by ``python setup.py build_ext --inplace``.  On
a machine with a GPU, every CUDA op goes through it; there is no silent
PyTorch fallback for CUDA tensors, so a missing or stale build fails loudly.
CPU tensors take the host code paths (which double as the test oracles).
"""
from __future__ import annotations

import importlib

_core = None
_err: Exception | None = None


def core():
    """Returns the imported ``turbol_core`` module or raises ImportError."""
    global _core, _err
    if _core is not None:
        return _core
    try:
        _core = importlib.import_module("turbol_b200.turbol_core")
    except Exception as e:  # pragma: no cover - exercised only without a build
        _err = e
        raise ImportError(
            "turbol_b200 native core is not built; run `python setup.py build_ext --inplace` "
            f"from the repository root ({e})"
        ) from e
    return _core


def ops():
    """The raw kernel launchers (``turbol_core.ops``)."""
    return core().ops


def require_cuda(t, what: str = "tensor"):
    """Raises unless ``t`` lives on a CUDA device (kernels never run on CPU)."""
    if not getattr(t, "is_cuda", False):
        raise ValueError(f"{what} must be a CUDA tensor for the sm_100a kernel path")
    return t
