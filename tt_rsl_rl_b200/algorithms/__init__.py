"""Learning algorithms (same names as ``rsl_rl.algorithms``)."""

from .distillation import Distillation
from .ppo import PPO

__all__ = ["PPO", "Distillation"]
