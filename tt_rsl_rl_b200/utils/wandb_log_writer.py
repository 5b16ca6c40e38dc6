"""Weights & Biases writer (``rsl_rl/utils/wandb_log_writer.py``); ``wandb`` is imported on construction."""

from __future__ import annotations

import os
import pathlib

from .log_writer import LogWriter


class WandbLogWriter(LogWriter):
    def __init__(self, log_dir: str, project_name: str | None = None, entity: str | None = None,
                 run_name: str | None = None, **kwargs) -> None:
        try:
            import wandb  # type: ignore
        except ImportError as exc:
            raise ImportError("WandbLogWriter requires the 'wandb' package") from exc
        self._wandb = wandb
        project = project_name or os.environ.get("WANDB_PROJECT", "tt_rsl_rl_b200")
        entity = entity or os.environ.get("WANDB_USERNAME")
        wandb.init(project=project, entity=entity, name=run_name or os.path.basename(log_dir), dir=log_dir, **kwargs)
        self.log_dir = log_dir

    def add_scalar(self, tag: str, scalar_value: float, global_step: int) -> None:
        self._wandb.log({tag: scalar_value}, step=global_step)

    def store_config(self, env_cfg, train_cfg: dict) -> None:
        self._wandb.config.update({"runner_cfg": train_cfg, "env_cfg": env_cfg if isinstance(env_cfg, dict) else
                                   repr(env_cfg)}, allow_val_change=True)

    def save_model(self, model_path: str, it: int) -> None:
        self._wandb.save(model_path, base_path=os.path.dirname(model_path))

    def save_file(self, path: str) -> None:
        self._wandb.save(path, base_path=os.path.dirname(path))

    def save_video(self, video: pathlib.Path, it: int) -> None:
        self._wandb.log({"Video": self._wandb.Video(str(video), format="mp4")}, step=it)

    def stop(self) -> None:
        self._wandb.finish()

    def abort(self) -> None:
        self._wandb.finish(exit_code=1)
