"""Replica-divergence detection for data-parallel training.

Every ``replica_check_interval`` updates each rank hashes its trainable parameters (an fp64 sum and a
position-weighted fp64 sum over the flat vector, so reorderings and sign flips change it), the hashes are all-gathered
over the process group and every rank compares them. All ranks raise :class:`ReplicaDivergenceError` together when
any hash differs, so no rank is left waiting in a later collective. With the fused engines the replicas are expected
to be bit-identical (rank-ordered reduction); on the PyTorch path the averaged gradients are identical on every rank
as well, so the check is exact there too.

The reference counterpart checks the maximum difference between chip replicas every k updates
(``rsl_rl_tt/ppo.py:684-698``); here the comparison is of hashes, so only 16 bytes per rank cross the network.
"""

from __future__ import annotations

import torch

from .errors import ReplicaDivergenceError


def parameter_hash(params) -> torch.Tensor:
    """fp64 ``[sum, sum(x_i * sin(i))]`` over the concatenation of ``params`` (on their device)."""
    flat = torch.cat([p.detach().reshape(-1) for p in params]).double()
    w = torch.arange(flat.numel(), device=flat.device, dtype=torch.float64).sin_()
    return torch.stack([flat.sum(), (flat * w).sum()])


class ReplicaChecker:
    """Calls :func:`check` every ``interval`` updates (``interval <= 0`` disables it)."""

    def __init__(self, interval: int, world_size: int) -> None:
        self.interval = int(interval)
        self.world_size = int(world_size)
        self.updates = 0

    def step(self, params) -> None:
        if self.interval <= 0 or self.world_size <= 1:
            return
        self.updates += 1
        if self.updates % self.interval == 0:
            check(params, self.updates)


def check(params, update: int | None = None) -> None:
    """All-gather the parameter hash of every rank and raise on every rank if they are not all equal."""
    h = parameter_hash(params)
    world = torch.distributed.get_world_size()
    gathered = [torch.zeros_like(h) for _ in range(world)]
    torch.distributed.all_gather(gathered, h)
    ref = gathered[0]
    bad = [r for r, g in enumerate(gathered) if not torch.equal(g, ref)]
    if bad:
        where = "" if update is None else f" after update {update}"
        raise ReplicaDivergenceError(f"parameter replicas diverged{where}: ranks {bad} differ from rank 0")
