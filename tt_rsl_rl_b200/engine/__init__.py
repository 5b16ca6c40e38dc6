"""Fused CUDA execution engines for the algorithms (device-resident state, sm_100a kernels, CUDA graphs)."""

from .distillation_engine import DistillationEngine, RecurrentDistillationEngine
from .ppo_engine import PPOEngine
from .recurrent_engine import RecurrentPPOEngine

__all__ = ["DistillationEngine", "PPOEngine", "RecurrentDistillationEngine", "RecurrentPPOEngine"]
