"""Environment interface and the synthetic benchmark environment."""

from .linear_gaussian import LinearGaussianVecEnv, humanoid_like
from .vec_env import VecEnv

__all__ = ["LinearGaussianVecEnv", "VecEnv", "humanoid_like"]
