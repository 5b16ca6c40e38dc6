"""Helpers (same names as ``rsl_rl.utils``) plus the framework's TensorDict."""

from .log_writer import CsvLogWriter, LogWriter
from .neptune_log_writer import NeptuneLogWriter
from .tensordict import TensorDict
from .utils import (
    check_nan,
    compile_model,
    get_param,
    reduce_gradients_in_buckets,
    resolve_callable,
    resolve_class,
    resolve_nn_activation,
    resolve_obs_groups,
    resolve_optimizer,
    split_and_pad_trajectories,
    unpad_trajectories,
)
from .wandb_log_writer import WandbLogWriter

__all__ = [
    "CsvLogWriter",
    "LogWriter",
    "NeptuneLogWriter",
    "TensorDict",
    "WandbLogWriter",
    "check_nan",
    "compile_model",
    "get_param",
    "reduce_gradients_in_buckets",
    "resolve_callable",
    "resolve_class",
    "resolve_nn_activation",
    "resolve_obs_groups",
    "resolve_optimizer",
    "split_and_pad_trajectories",
    "unpad_trajectories",
]
