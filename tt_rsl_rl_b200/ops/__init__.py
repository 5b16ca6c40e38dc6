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
_COUNTER: list[int] | None = None

# Entry points that launch kernels (the rest are host-side planning, sizing and IPC helpers).
LAUNCHING = frozenset({
    "adam_step", "adv_gather_stats", "adv_normalize", "colstats", "counter_add", "gae", "gather_minibatch",
    "gaussian_sample", "gemm", "lg_env_step", "mse_grad", "norm_update", "p2p_allreduce_f64", "p2p_broadcast_f32",
    "ppo_loss", "prep_obs", "process_step", "reduce_segments", "rnd_intrinsic", "rnd_reward_scale", "rnn_cell_bwd",
    "rnn_cell_fwd", "rnn_mask", "to_bf16_padded",
})


class _CountingModule:
    """Forwards to the extension and counts calls of kernel-launching entry points."""

    def __init__(self, mod) -> None:
        self._mod = mod

    def __getattr__(self, name: str):
        fn = getattr(self._mod, name)
        if name not in LAUNCHING:
            return fn

        def counted(*args, **kwargs):
            if _COUNTER is not None:
                _COUNTER[0] += 1
            return fn(*args, **kwargs)

        return counted


class count_launches:
    """Context manager counting this framework's kernel launches issued from Python (``.n`` after exit).

    A CUDA-graph replay launches exactly the kernels recorded while it was captured, so counting one eager
    iteration gives the launches of a replayed one.
    """

    def __init__(self) -> None:
        self.n = 0

    def __enter__(self) -> count_launches:
        global _COUNTER
        _COUNTER = [0]
        return self

    def __exit__(self, *exc) -> None:
        global _COUNTER
        self.n = _COUNTER[0]
        _COUNTER = None


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
    if _COUNTER is not None:
        return _CountingModule(_EXT)
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
