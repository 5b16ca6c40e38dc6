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
_PROFILER: profile_ops | None = None

# Entry points that launch kernels (the rest are host-side planning, sizing and IPC helpers).
LAUNCHING = frozenset({
    "adam_step", "adv_gather_stats", "adv_normalize", "colstats", "counter_add", "gae", "gather_minibatch",
    "gaussian_sample", "gemm", "lg_env_step", "mse_grad", "norm_update", "p2p_allreduce_f64", "p2p_broadcast_f32",
    "ppo_loss", "prep_obs", "process_step", "reduce_segments", "rnd_intrinsic", "rnd_reward_scale", "rnn_cell_bwd",
    "rnn_cell_fwd", "rnn_mask", "to_bf16_padded",
})


class _CountingModule:
    """Forwards to the extension; counts (and, under :class:`profile_ops`, times) calls of kernel-launching entry
    points."""

    def __init__(self, mod) -> None:
        self._mod = mod

    def __getattr__(self, name: str):
        fn = getattr(self._mod, name)
        if name not in LAUNCHING:
            return fn

        def counted(*args, **kwargs):
            if _COUNTER is not None:
                _COUNTER[0] += 1
            prof = _PROFILER
            if prof is not None:
                return prof._timed(name, fn, args, kwargs)
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


class profile_ops:
    """Context manager timing every kernel-launching entry point called from Python.

    Each call is bracketed by CUDA events on the current stream; the events are resolved when the block exits (one
    synchronisation, no per-call host wait), so a time is the device time of that call's kernels. ``.stats[name] =
    [calls, total_ms]``; :meth:`table` lists them by total time. Calls made while a CUDA graph is being captured are
    not timed (a replay is one graph launch): profile eager iterations (``b200_cfg["graphs"] = False``, or the first
    iteration of a captured path). The reference plugin's op profiler has the same role with a device
    synchronisation around every op (``scripts/profile_ops.py``).
    """

    def __init__(self, event_factory=None, synchronize=None, capturing=None) -> None:
        self._event = event_factory or (lambda: torch.cuda.Event(enable_timing=True))
        self._sync = synchronize or torch.cuda.synchronize
        self._capturing = capturing or torch.cuda.is_current_stream_capturing
        self._pending: list = []
        self.stats: dict[str, list] = {}

    def _timed(self, name: str, fn, args, kwargs):
        if self._capturing():
            return fn(*args, **kwargs)
        start, end = self._event(), self._event()
        start.record()
        out = fn(*args, **kwargs)
        end.record()
        self._pending.append((name, start, end))
        return out

    def __enter__(self) -> profile_ops:
        global _PROFILER
        if _PROFILER is not None:
            raise RuntimeError("profile_ops blocks do not nest")
        self._pending = []
        _PROFILER = self
        return self

    def __exit__(self, *exc) -> None:
        global _PROFILER
        _PROFILER = None
        self._sync()
        for name, start, end in self._pending:
            entry = self.stats.setdefault(name, [0, 0.0])
            entry[0] += 1
            entry[1] += start.elapsed_time(end)
        self._pending = []

    def table(self) -> list[dict]:
        """One row per entry point: calls, total milliseconds, mean microseconds, share of the total."""
        total = sum(ms for _, ms in self.stats.values()) or 1.0
        rows = [{"op": k, "calls": c, "total_ms": round(ms, 4), "mean_us": round(1e3 * ms / c, 2),
                 "share": round(ms / total, 4)} for k, (c, ms) in self.stats.items()]
        return sorted(rows, key=lambda r: -r["total_ms"])


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
    if _COUNTER is not None or _PROFILER is not None:
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
