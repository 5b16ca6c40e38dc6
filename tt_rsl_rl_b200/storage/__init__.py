"""Rollout storage (same names as ``rsl_rl.storage``)."""

from .rollout_storage import RolloutStorage

__all__ = ["RolloutStorage"]
