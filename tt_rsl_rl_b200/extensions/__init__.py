"""Extensions of the learning algorithms (same names as ``rsl_rl.extensions``)."""

from .rnd import RandomNetworkDistillation, resolve_rnd_config
from .symmetry import Symmetry, resolve_symmetry_config

__all__ = ["RandomNetworkDistillation", "Symmetry", "resolve_rnd_config", "resolve_symmetry_config"]
