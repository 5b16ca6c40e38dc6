"""Runners (same names as ``rsl_rl.runners``)."""

from .distillation_runner import DistillationRunner
from .on_policy_runner import OnPolicyRunner

__all__ = ["DistillationRunner", "OnPolicyRunner"]
