"""Turn the agent configuration of a simulator host into the configuration of a training run of this framework.

A simulator host (e.g. Isaac Lab) trains with ``OnPolicyRunner(env, agent_cfg.to_dict(), log_dir, device)``. When it
serves its environments over the bridge instead (:class:`~tt_rsl_rl_b200.env.bridge.EnvServer` with ``agent_cfg=``),
the learner receives that dictionary (``RemoteVecEnv.agent_cfg``) or reads the saved ``params/agent.yaml``
(:func:`load_agent_cfg`). :func:`b200_agent_cfg` makes the only changes that define this backend: class names that point
into upstream ``rsl_rl`` are mapped to this package's classes of the same name, the algorithm gets its ``b200_cfg``
options, and optionally a CSV log writer; network sizes, learning rates, ``obs_groups`` and everything else stay as the
host set them, so both runs are the same experiment.

The reference plugin does the same for its own backend (``rsl_rl_tt/bridge/config.py:36-55``).
"""

from __future__ import annotations

import copy
import json
from pathlib import Path
from typing import Any

CSV_WRITER = "tt_rsl_rl_b200.utils.log_writer:CsvLogWriter"
_RUNNERS = ("OnPolicyRunner", "DistillationRunner")
_ALGORITHMS = {"OnPolicyRunner": "PPO", "DistillationRunner": "Distillation"}


def load_agent_cfg(path: str | Path) -> dict:
    """A saved agent configuration: JSON, or YAML (Isaac Lab's ``params/agent.yaml``; its Python tags for tuples and
    slices are read with the full loader)."""
    path = Path(path)
    text = path.read_text()
    if path.suffix.lower() in (".yaml", ".yml"):
        import yaml

        loaded = yaml.unsafe_load(text) if "!!python" in text else yaml.safe_load(text)
    else:
        loaded = json.loads(text)
    if not isinstance(loaded, dict):
        raise ValueError(f"{path}: an agent configuration must be a mapping, got {type(loaded).__name__}")
    return loaded


def _own_class_name(name: Any) -> Any:
    """``"rsl_rl.<module>:<Class>"`` or ``"rsl_rl.<module>.<Class>"`` -> ``"<Class>"`` (resolved in this package)."""
    if not isinstance(name, str) or not name.startswith("rsl_rl."):
        return name
    return name.rsplit(":", 1)[-1] if ":" in name else name.rsplit(".", 1)[-1]


def _map_class_names(node: Any) -> Any:
    if isinstance(node, dict):
        return {k: (_own_class_name(v) if k == "class_name" else _map_class_names(v)) for k, v in node.items()}
    if isinstance(node, list):
        return [_map_class_names(v) for v in node]
    return node


def b200_agent_cfg(agent_cfg: dict[str, Any], *, device: str = "cuda:0", engine: str = "auto", graphs: bool = True,
                   csv_log: bool = False, extra_b200_cfg: dict | None = None) -> dict:
    """The runner configuration of this framework's run for ``agent_cfg`` (a copy; the argument is not changed).

    The device is returned in ``cfg["device"]`` for convenience; ``OnPolicyRunner`` takes it as its own argument."""
    cfg = copy.deepcopy(agent_cfg)
    runner = cfg.get("class_name", "OnPolicyRunner")
    if runner not in _RUNNERS:
        raise NotImplementedError(f"runner {runner!r}: supported runners are {_RUNNERS}")
    models = ("student", "teacher") if runner == "DistillationRunner" else ("actor", "critic")
    missing = [k for k in ("algorithm", "obs_groups", *models) if k not in cfg]
    if missing:
        raise ValueError(f"the agent configuration has no {missing}: this framework reads the rsl_rl v5 format "
                         f"(separate models per role and obs_groups); got keys {sorted(cfg)}")
    cfg = _map_class_names(cfg)
    algorithm = cfg["algorithm"]
    want = _ALGORITHMS[runner]
    if algorithm.get("class_name", want) != want:
        raise NotImplementedError(f"algorithm {algorithm['class_name']!r} with {runner}: expected {want}")
    algorithm["class_name"] = want
    algorithm["b200_cfg"] = {"engine": engine, "graphs": bool(graphs), **(extra_b200_cfg or {})}
    cfg["device"] = str(device)
    if csv_log:
        cfg["logger"] = {"class_name": CSV_WRITER}
    return cfg


__all__ = ["CSV_WRITER", "b200_agent_cfg", "load_agent_cfg"]
