"""Fused CUDA execution engines for the algorithms (device-resident state, sm_100a kernels, CUDA graphs)."""

from .ppo_engine import PPOEngine

__all__ = ["PPOEngine"]
