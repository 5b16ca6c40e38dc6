"""Neptune writer (``rsl_rl/utils/neptune_log_writer.py``); ``neptune`` is imported on construction."""

from __future__ import annotations

import os
import pathlib

from .log_writer import LogWriter


class NeptuneLogWriter(LogWriter):
    def __init__(self, log_dir: str, project_name: str | None = None, run_name: str | None = None, **kwargs) -> None:
        try:
            import neptune  # type: ignore
        except ImportError as exc:
            raise ImportError("NeptuneLogWriter requires the 'neptune' package") from exc
        project = project_name or os.environ.get("NEPTUNE_PROJECT")
        self.run = neptune.init_run(project=project, name=run_name or os.path.basename(log_dir), **kwargs)
        self.log_dir = log_dir

    def add_scalar(self, tag: str, scalar_value: float, global_step: int) -> None:
        self.run[tag].append(scalar_value, step=global_step)

    def store_config(self, env_cfg, train_cfg: dict) -> None:
        self.run["runner_cfg"] = repr(train_cfg)
        self.run["env_cfg"] = repr(env_cfg)

    def save_model(self, model_path: str, it: int) -> None:
        self.run[f"model/saved_model_{it}"].upload(model_path)

    def save_file(self, path: str) -> None:
        self.run[f"files/{os.path.basename(path)}"].upload(path)

    def save_video(self, video: pathlib.Path, it: int) -> None:
        self.run[f"videos/{video.name}"].upload(str(video))

    def stop(self) -> None:
        self.run.stop()
