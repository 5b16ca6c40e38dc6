"""Environment interface, the synthetic benchmark environment and the remote environment bridge."""

from .bridge import EnvServer, RemoteEnvError, RemoteEnvTimeoutError, RemoteVecEnv
from .classic import BatchedCartPole, BatchedCartPolePO, BatchedPendulum, Tracking12
from .linear_gaussian import LinearGaussianVecEnv, humanoid_like
from .vec_env import VecEnv

__all__ = ["BatchedCartPole", "BatchedCartPolePO", "BatchedPendulum", "EnvServer", "LinearGaussianVecEnv",
           "RemoteEnvError", "RemoteEnvTimeoutError", "RemoteVecEnv", "Tracking12", "VecEnv", "humanoid_like"]
