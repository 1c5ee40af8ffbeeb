"""Loader of the in-tree sm_100a extension ``vllm_neuron_b200._C``.

CUDA tensors always go to the compiled kernels.  If the extension is missing, the first CUDA
op raises instead of silently falling back to PyTorch; CPU tensors use the fp32 torch
references (the oracle used by the tests and by CPU plumbing runs).
"""
from __future__ import annotations

import importlib
import os

_C = None
_ERR: Exception | None = None


def ext():
    """Return the compiled extension module, raising a clear error if it is unavailable."""
    global _C, _ERR
    if _C is not None:
        return _C
    if _ERR is not None:
        raise _ERR
    try:
        _C = importlib.import_module("vllm_neuron_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = RuntimeError(
            "vllm_neuron_b200._C (sm_100a kernels) is not built or failed to load: "
            f"{e!r}. Build it with `python setup.py build_ext --inplace` in the repo root."
        )
        raise _ERR from e
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except Exception:
        return False


def so_path() -> str | None:
    try:
        return os.path.abspath(ext().__file__)
    except Exception:
        return None
