"""Environment interface, the synthetic benchmark environment and the remote environment bridge."""

from .agent_cfg import b200_agent_cfg, load_agent_cfg
from .bridge import EnvServer, RemoteEnvError, RemoteEnvTimeoutError, RemoteVecEnv
from .classic import ENV_CLASSES, BatchedCartPole, BatchedCartPolePO, BatchedPendulum, Tracking12, make_env
from .linear_gaussian import LinearGaussianVecEnv, humanoid_like
from .vec_env import VecEnv

__all__ = ["ENV_CLASSES", "BatchedCartPole", "BatchedCartPolePO", "BatchedPendulum", "EnvServer", "LinearGaussianVecEnv",
           "RemoteEnvError", "RemoteEnvTimeoutError", "RemoteVecEnv", "Tracking12", "VecEnv", "b200_agent_cfg",
           "humanoid_like", "load_agent_cfg", "make_env"]
