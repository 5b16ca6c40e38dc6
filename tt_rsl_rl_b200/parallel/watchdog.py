"""Host-side failure detection for data-parallel runs.

Every rank publishes a heartbeat (its iteration number) to the rendezvous key-value store once per iteration and,
before launching work that waits on peers (the gradient exchange), checks that every peer has reached the same
iteration. A rank that crashed, exited or hangs between iterations is reported within ``timeout_s`` as
:class:`CommTimeoutError` instead of leaving the others blocked in a collective. The device-side exchange has its own
bounded waits for failures inside an iteration.

Upstream rsl_rl has no failure detection (a dead rank blocks NCCL until its timeout); this is an addition.
"""

from __future__ import annotations

import time

from .errors import CommTimeoutError


class RankWatchdog:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 60.0, prefix: str = "tt_rsl_rl_b200/hb") -> None:
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = timeout_s
        self.prefix = prefix

    @classmethod
    def from_default_group(cls, timeout_s: float = 60.0) -> RankWatchdog:
        import torch.distributed as dist
        from torch.distributed import distributed_c10d

        store = distributed_c10d._get_default_store()
        return cls(store, dist.get_rank(), dist.get_world_size(), timeout_s)

    def _key(self, rank: int) -> str:
        return f"{self.prefix}/{rank}"

    def beat(self, iteration: int) -> None:
        self.store.set(self._key(self.rank), str(iteration))

    def check(self, iteration: int) -> None:
        """Return once every rank has published ``iteration`` (or later); raise after ``timeout_s``."""
        deadline = time.monotonic() + self.timeout_s
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            still = []
            for r in pending:
                try:
                    raw = self.store.get(self._key(r)) if self._has(r) else None
                except Exception:
                    raw = None
                if raw is None or int(raw) < iteration:
                    still.append(r)
            pending = still
            if not pending:
                return
            if time.monotonic() > deadline:
                raise CommTimeoutError(
                    f"rank {self.rank}: ranks {pending} did not reach iteration {iteration} within {self.timeout_s}s"
                )
            time.sleep(0.01)

    def _has(self, rank: int) -> bool:
        try:
            return bool(self.store.check([self._key(rank)]))
        except Exception:
            return False
