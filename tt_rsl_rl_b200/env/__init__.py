"""Environment interface, the synthetic benchmark environment and the remote environment bridge."""

from .bridge import EnvServer, RemoteEnvError, RemoteEnvTimeoutError, RemoteVecEnv
from .linear_gaussian import LinearGaussianVecEnv, humanoid_like
from .vec_env import VecEnv

__all__ = ["EnvServer", "LinearGaussianVecEnv", "RemoteEnvError", "RemoteEnvTimeoutError", "RemoteVecEnv", "VecEnv",
           "humanoid_like"]
