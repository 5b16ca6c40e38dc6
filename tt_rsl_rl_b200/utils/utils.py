"""Configuration resolution and tensor helpers shared by the whole framework.

Behaviour follows rsl_rl v5.5.2 (``rsl_rl/utils/utils.py``): the same names, accepted strings and error cases, so that
configurations written for rsl_rl resolve identically here.
"""

from __future__ import annotations

import copy
import importlib
import warnings
from collections.abc import Callable, Iterable
from typing import Any

import torch

from .tensordict import TensorDict, is_tensordict


def get_param(param: Any, idx: int) -> Any:
    """Element ``idx`` of a list/tuple parameter, or the parameter itself when it is a scalar."""
    return param[idx] if isinstance(param, (tuple, list)) else param


_ACTIVATIONS: dict[str, Callable[[], torch.nn.Module]] = {
    "elu": torch.nn.ELU,
    "selu": torch.nn.SELU,
    "relu": torch.nn.ReLU,
    "crelu": torch.nn.CELU,
    "lrelu": torch.nn.LeakyReLU,
    "tanh": torch.nn.Tanh,
    "sigmoid": torch.nn.Sigmoid,
    "softplus": torch.nn.Softplus,
    "gelu": torch.nn.GELU,
    "swish": torch.nn.SiLU,
    "mish": torch.nn.Mish,
    "identity": torch.nn.Identity,
}


def resolve_nn_activation(act_name: str) -> torch.nn.Module:
    """Activation module for a name (``rsl_rl/utils/utils.py:34-68``); raises ``ValueError`` for unknown names."""
    key = act_name.lower()
    if key not in _ACTIVATIONS:
        raise ValueError(f"Invalid activation function '{act_name}'. Valid activations are: {list(_ACTIVATIONS)}")
    return _ACTIVATIONS[key]()


_OPTIMIZERS: dict[str, type] = {
    "adam": torch.optim.Adam,
    "adamw": torch.optim.AdamW,
    "sgd": torch.optim.SGD,
    "rmsprop": torch.optim.RMSprop,
}


def resolve_optimizer(optimizer_name: str) -> type:
    """Optimizer class for a name (``rsl_rl/utils/utils.py:71-96``)."""
    key = optimizer_name.lower()
    if key not in _OPTIMIZERS:
        raise ValueError(f"Invalid optimizer '{optimizer_name}'. Valid optimizers are: {list(_OPTIMIZERS)}")
    return _OPTIMIZERS[key]


def _lookup_attr(obj: Any, dotted: str) -> Any:
    for part in dotted.split("."):
        obj = getattr(obj, part)
    return obj


# Packages searched for bare class names, in order (the public API of the framework).
_SEARCH_PACKAGES = (
    "tt_rsl_rl_b200.algorithms",
    "tt_rsl_rl_b200.models",
    "tt_rsl_rl_b200.modules",
    "tt_rsl_rl_b200.extensions",
    "tt_rsl_rl_b200.runners",
    "tt_rsl_rl_b200.storage",
    "tt_rsl_rl_b200.env",
    "tt_rsl_rl_b200.utils",
)


def resolve_callable(callable_or_name: type | Callable | str) -> Callable:
    """Resolve a callable given directly, as ``"pkg.mod:Attr.Sub"``, as ``"pkg.mod.Attr"`` or as a bare name.

    Bare names are searched in the modules of this package (the role ``rsl_rl`` plays in ``rsl_rl/utils/utils.py:99``),
    so ``"PPO"``, ``"MLPModel"`` or ``"GaussianDistribution"`` resolve to this framework's classes.
    """
    if callable(callable_or_name):
        return callable_or_name
    if not isinstance(callable_or_name, str):
        raise TypeError(f"Expected callable or string, got {type(callable_or_name)}")
    name = callable_or_name
    if ":" in name:
        module_path, attr_path = name.rsplit(":", 1)
        return _lookup_attr(importlib.import_module(module_path), attr_path)
    if "." in name:
        parts = name.split(".")
        found_module = False
        # try the longest importable module prefix first
        for cut in range(len(parts) - 1, 0, -1):
            try:
                module = importlib.import_module(".".join(parts[:cut]))
            except ModuleNotFoundError:
                continue
            found_module = True
            try:
                return _lookup_attr(module, ".".join(parts[cut:]))
            except AttributeError:
                continue
        if found_module:
            raise AttributeError(f"Could not resolve '{name}': attribute not found in module")
        raise ImportError(f"Could not resolve '{name}': no valid module.attr split found")
    for package in _SEARCH_PACKAGES:
        module = importlib.import_module(package)
        if hasattr(module, name):
            return getattr(module, name)
    raise ValueError(
        f"Could not resolve '{name}'. Use qualified name like 'module.path:ClassName' or pass the class directly."
    )


def resolve_class(cfg: dict) -> tuple[Callable, dict]:
    """``(class, kwargs)`` from a config dict with a ``class_name`` key; ``cfg`` itself is not modified."""
    kwargs = copy.deepcopy(cfg)
    return resolve_callable(kwargs.pop("class_name")), kwargs


def resolve_obs_groups(obs: Any, obs_groups: dict[str, list[str]], default_sets: list[str]) -> dict[str, list[str]]:
    """Validate ``obs_groups`` against the environment's observations and fill missing default sets.

    Rules (``rsl_rl/utils/utils.py:192-287``): every listed group must exist and no set may be empty; a missing default
    set takes the group of the same name if present, else the ``"policy"`` group, else it is an error.
    """
    if len(obs_groups) == 0:
        warnings.warn(
            "The observation configuration dictionary 'obs_groups' is empty and thus likely not configured. Consider"
            " configuring the 'obs_groups' dictionary explicitly"
        )
    for set_name, groups in obs_groups.items():
        if len(groups) == 0:
            raise ValueError(f"The '{set_name}' key in the 'obs_groups' dictionary can not be an empty list.")
        for group in groups:
            if group not in obs:
                raise ValueError(
                    f"Observation '{group}' in observation set '{set_name}' not found in the observations from the"
                    f" environment. Available observations from the environment: {list(obs.keys())}"
                )
    for set_name in default_sets:
        if set_name in obs_groups:
            continue
        if set_name in obs:
            fallback = set_name
        elif "policy" in obs:
            fallback = "policy"
        else:
            raise ValueError(
                f"The observation configuration dictionary 'obs_groups' does not contain the '{set_name}' key and no"
                " suitable observation could be found in the observations from the environment. Please refer to"
                " `resolve_obs_groups()` for information on how to configure the 'obs_groups' dictionary correctly."
            )
        obs_groups[set_name] = [fallback]
        warnings.warn(
            f"The observation configuration dictionary 'obs_groups' does not contain the '{set_name}' key. Using the"
            f" observation group '{fallback}' for it. Consider adding the '{set_name}' key to 'obs_groups'."
        )
    print("-" * 80)
    print("Resolved observation sets: ")
    for set_name, groups in obs_groups.items():
        print("\t", set_name, ": ", groups)
    print("-" * 80)
    return obs_groups


def _non_finite_kind(t: torch.Tensor) -> str:
    has_nan = bool(torch.isnan(t).any())
    has_inf = bool(torch.isinf(t).any())
    return "NaN and Inf" if has_nan and has_inf else "NaN" if has_nan else "Inf"


def check_nan(obs: Any, rewards: torch.Tensor, dones: torch.Tensor) -> None:
    """Raise ``ValueError`` if observations, rewards or dones contain NaN/Inf (``rsl_rl/utils/utils.py:290``)."""
    for key, tensor in obs.items():
        if not torch.isfinite(tensor).all():
            raise ValueError(
                f"The observation group '{key}' returned by the environment contains {_non_finite_kind(tensor)}"
                " values. This usually indicates a bug in the environment's step() or reset() function."
            )
    if not torch.isfinite(rewards).all():
        raise ValueError(
            f"The rewards returned by the environment contain {_non_finite_kind(rewards)} values. This usually"
            " indicates a bug in the environment's reward computation."
        )
    if not torch.isfinite(dones).all():
        raise ValueError(
            f"The dones returned by the environment contain {_non_finite_kind(dones)} values. This usually indicates"
            " a bug in the environment's termination logic."
        )


def compile_model(model: torch.nn.Module, mode: str | None = None) -> torch.nn.Module:
    """Optionally wrap a model in ``torch.compile`` (off by default; never used on the fused CUDA path).

    CUDA-graph compile modes are rejected as in ``rsl_rl/utils/utils.py:319-342``.
    """
    if mode is None:
        return model
    if mode in ("reduce-overhead", "max-autotune"):
        raise ValueError(
            f"torch_compile_mode='{mode}' uses CUDA graphs which are incompatible with the algorithms' multi-model "
            "forward pattern. Use 'default' or 'max-autotune-no-cudagraphs', or set to None to disable."
        )
    return torch.compile(model, mode=mode)  # type: ignore[return-value]


def reduce_gradients_in_buckets(params: Iterable[torch.nn.Parameter], world_size: int, bucket_mb: float) -> None:
    """Average gradients over ``torch.distributed`` ranks in buckets of at most ``bucket_mb`` MiB.

    Used by the PyTorch (CPU / gloo) path; the CUDA path reduces gradients inside the fused optimizer kernel.
    Small gradients are packed into one buffer per bucket; a gradient larger than a bucket is reduced in slices
    (``rsl_rl/utils/utils.py:345-392``).
    """
    limit = int(bucket_mb * 1024 * 1024)
    grads = [p.grad.view(-1) for p in params if p.grad is not None]
    i = 0
    while i < len(grads):
        g = grads[i]
        if g.numel() * g.element_size() > limit:
            step = max(1, limit // g.element_size())
            for off in range(0, g.numel(), step):
                chunk = g.narrow(0, off, min(step, g.numel() - off))
                torch.distributed.all_reduce(chunk, op=torch.distributed.ReduceOp.SUM)
                chunk /= world_size
            i += 1
            continue
        j, used = i, 0
        while j < len(grads) and used + grads[j].numel() * grads[j].element_size() <= limit:
            used += grads[j].numel() * grads[j].element_size()
            j += 1
        packed = torch.cat(grads[i:j])
        torch.distributed.all_reduce(packed, op=torch.distributed.ReduceOp.SUM)
        packed /= world_size
        off = 0
        for g2 in grads[i:j]:
            g2.copy_(packed[off : off + g2.numel()])
            off += g2.numel()
        i = j


def _trajectory_lengths(dones: torch.Tensor) -> torch.Tensor:
    """Lengths of the trajectories obtained by cutting each env's time series after every done (env-major order)."""
    d = dones.clone().reshape(dones.shape[0], dones.shape[1])
    d[-1] = 1
    flat = d.transpose(1, 0).reshape(-1)
    ends = torch.nonzero(flat, as_tuple=False)[:, 0]
    starts = torch.cat((ends.new_tensor([-1]), ends[:-1]))
    return ends - starts


def _pad_split(tensor: torch.Tensor, lengths: list[int]) -> torch.Tensor:
    T = tensor.shape[0]
    pieces = list(torch.split(tensor.transpose(1, 0).flatten(0, 1), lengths))
    # a zero trajectory of full length guarantees the padded time axis is T long
    pieces.append(tensor.new_zeros(T, *tensor.shape[2:]))
    padded = torch.nn.utils.rnn.pad_sequence(pieces)
    return padded[:, :-1]


def split_and_pad_trajectories(tensor: torch.Tensor | TensorDict, dones: torch.Tensor):
    """Cut ``[T, N, ...]`` data into trajectories at dones and zero-pad them to length T.

    Returns ``(padded [T, num_traj, ...], masks [T, num_traj])`` with trajectories ordered env by env, as
    ``rsl_rl/utils/utils.py:395-446``.
    """
    lengths_t = _trajectory_lengths(dones)
    lengths = lengths_t.tolist()
    T = tensor.shape[0]
    if is_tensordict(tensor):
        padded = {k: _pad_split(v, lengths) for k, v in tensor.items()}
        out = TensorDict(padded, batch_size=[T, len(lengths)], device=tensor.device)
    else:
        out = _pad_split(tensor, lengths)
    masks = lengths_t > torch.arange(0, T, device=lengths_t.device).unsqueeze(1)
    return out, masks


def unpad_trajectories(trajectories: torch.Tensor | TensorDict, masks: torch.Tensor):
    """Inverse of :func:`split_and_pad_trajectories`: back to ``[T, N, ...]``."""
    T = trajectories.shape[0]
    valid = trajectories.transpose(1, 0)[masks.transpose(1, 0)]
    if is_tensordict(trajectories):
        return valid.view(-1, T).transpose(1, 0)
    return valid.view(-1, T, *trajectories.shape[2:]).transpose(1, 0)
