"""Runners (same names as ``rsl_rl.runners``)."""

from .distillation_runner import DistillationRunner
from .on_policy_runner import OnPolicyRunner, latest_checkpoint

__all__ = ["DistillationRunner", "OnPolicyRunner", "latest_checkpoint"]
