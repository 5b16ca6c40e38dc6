"""sm_100a CUDA kernels of the framework.

The compiled extension ``tt_rsl_rl_b200._C`` is built in-tree by ``python setup.py build_ext --inplace``. On a machine
with a CUDA device the kernels are the only compute path for CUDA tensors: :func:`ext` raises if the extension is
missing instead of falling back to PyTorch.
"""

from __future__ import annotations

import importlib

import torch

_EXT = None
_EXT_ERROR: Exception | None = None


def ext():
    """Return the compiled extension module, raising a clear error if it is not built."""
    global _EXT, _EXT_ERROR
    if _EXT is None and _EXT_ERROR is None:
        try:
            _EXT = importlib.import_module("tt_rsl_rl_b200._C")
        except Exception as exc:  # pragma: no cover - depends on the build
            _EXT_ERROR = exc
    if _EXT is None:
        raise RuntimeError(
            "tt_rsl_rl_b200._C is not built; run `python setup.py build_ext --inplace` in the repository root"
        ) from _EXT_ERROR
    return _EXT


def available() -> bool:
    """Whether the extension is importable and a CUDA device is present."""
    if not torch.cuda.is_available():
        return False
    try:
        ext()
    except RuntimeError:
        return False
    return True
