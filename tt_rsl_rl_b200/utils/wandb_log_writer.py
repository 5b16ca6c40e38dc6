"""Weights & Biases writer (``rsl_rl/utils/wandb_log_writer.py``): every scalar goes to TensorBoard files in the run
folder and to W&B; configurations, checkpoints, files and videos are uploaded. ``wandb`` is imported on construction.

Kept as upstream has them, since dashboards and scripts read them: the TensorBoard copy, the run name (the last
component of the log folder), the entity from ``WANDB_USERNAME``, the config keys ``train_cfg`` / ``env_cfg`` and the
video key ``video``.
"""

from __future__ import annotations

import os
import pathlib
from dataclasses import asdict, is_dataclass

from torch.utils.tensorboard import SummaryWriter

from .log_writer import LogWriter


def env_cfg_dict(env_cfg) -> dict | object:
    """An environment configuration as a plain dict where it has a conversion (``to_dict()``, a dataclass)."""
    if hasattr(env_cfg, "to_dict"):
        try:
            return env_cfg.to_dict()
        except Exception:  # a to_dict that fails keeps the object's text
            return repr(env_cfg)
    if is_dataclass(env_cfg) and not isinstance(env_cfg, type):
        return asdict(env_cfg)
    return env_cfg if isinstance(env_cfg, dict) else repr(env_cfg)


class WandbLogWriter(SummaryWriter, LogWriter):
    def __init__(self, log_dir: str, project_name: str | None = None, **kwargs) -> None:
        try:
            import wandb  # type: ignore
        except ImportError as exc:
            raise ModuleNotFoundError("WandbLogWriter requires the 'wandb' package") from exc
        super().__init__(log_dir, flush_secs=10)
        self._wandb = wandb
        wandb.init(project=project_name or os.environ.get("WANDB_PROJECT"), entity=os.environ.get("WANDB_USERNAME"),
                   name=os.path.split(log_dir.rstrip("/"))[-1], config={"log_dir": log_dir}, **kwargs)

    def add_scalar(self, tag: str, scalar_value: float, global_step: int | None = None, walltime: float | None = None,
                   new_style: bool = False) -> None:
        super().add_scalar(tag, scalar_value, global_step=global_step, walltime=walltime, new_style=new_style)
        self._wandb.log({tag: scalar_value}, step=global_step)

    def store_config(self, env_cfg, train_cfg: dict) -> None:
        self._wandb.config.update({"train_cfg": train_cfg})
        self._wandb.config.update({"env_cfg": env_cfg_dict(env_cfg)})

    def save_model(self, model_path: str, it: int) -> None:
        self._wandb.save(model_path, base_path=os.path.dirname(model_path))

    def save_file(self, path: str) -> None:
        self._wandb.save(path, base_path=os.path.dirname(path))

    def save_video(self, video: pathlib.Path, it: int) -> None:
        self._wandb.log({"video": self._wandb.Video(str(video), format="mp4")}, step=it)

    def stop(self) -> None:
        self.close()
        self._wandb.finish()

    def abort(self) -> None:
        self.close()
        self._wandb.finish(exit_code=1)
