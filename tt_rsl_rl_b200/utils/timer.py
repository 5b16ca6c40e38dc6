"""Section timing and host-transfer accounting (tracing / observability).

:class:`SectionTimer` brackets named sections with CUDA events on the current stream (no device synchronisation
inside the hot path; the events are resolved once per iteration, after the iteration's own host read) or with the
host clock on the CPU, and opens an NVTX range per section so an external timeline shows the same names. It does
nothing while a CUDA graph is being captured (event records would become graph nodes) and when disabled.

:class:`HostTransfers` counts the device-to-host reads the fused engines make (calls and bytes per tag), the
counterpart of the reference plugin's allow-list transfer counter (``rsl_rl_tt/tt_common.py:43-64``): the engines read
a handful of small tensors per iteration (loss statistics, status word, non-finite flag, learning rate) and never
anything of rollout size.
"""

from __future__ import annotations

import time
from collections import defaultdict
from contextlib import contextmanager

import torch


class SectionTimer:
    def __init__(self, enabled: bool = False, device: str | torch.device = "cpu") -> None:
        self.enabled = bool(enabled)
        self.cuda = torch.device(device).type == "cuda"
        self._pending: list[tuple[str, object, object]] = []
        self.totals: dict[str, float] = defaultdict(float)

    @contextmanager
    def section(self, name: str):
        if not self.enabled or (self.cuda and torch.cuda.is_current_stream_capturing()):
            yield
            return
        if self.cuda:
            torch.cuda.nvtx.range_push(name)
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            start.record()
            try:
                yield
            finally:
                stop.record()
                torch.cuda.nvtx.range_pop()
            self._pending.append((name, start, stop))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self._pending.append((name, t0, time.perf_counter()))

    def resolve(self) -> dict[str, float]:
        """Milliseconds per section name since the last call (waits for the last recorded event only)."""
        out: dict[str, float] = defaultdict(float)
        if self._pending:
            if self.cuda:
                self._pending[-1][2].synchronize()
                for name, a, b in self._pending:
                    out[name] += a.elapsed_time(b)
            else:
                for name, a, b in self._pending:
                    out[name] += (b - a) * 1e3
        self._pending.clear()
        for k, v in out.items():
            self.totals[k] += v
        return dict(out)


class HostTransfers:
    """Per-tag count and bytes of device-to-host reads (process-wide, cheap enough to stay on)."""

    calls: dict[str, int] = defaultdict(int)
    nbytes: dict[str, int] = defaultdict(int)

    @classmethod
    def read(cls, t: torch.Tensor, tag: str):
        """``t.tolist()``, recorded under ``tag``."""
        cls.calls[tag] += 1
        cls.nbytes[tag] += t.numel() * t.element_size()
        out = t.tolist()
        return out

    @classmethod
    def snapshot(cls) -> dict[str, int]:
        return {"calls": sum(cls.calls.values()), "bytes": sum(cls.nbytes.values())}

    @classmethod
    def reset(cls) -> None:
        cls.calls.clear()
        cls.nbytes.clear()
