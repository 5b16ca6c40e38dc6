"""Pluggable logging back ends (``rsl_rl/utils/log_writer.py``): only :meth:`LogWriter.add_scalar` is required."""

from __future__ import annotations

import csv
import json
import os
import pathlib
import time
from abc import ABC, abstractmethod


class LogWriter(ABC):
    @abstractmethod
    def add_scalar(self, tag: str, scalar_value: float, global_step: int) -> None:
        """Record one scalar."""

    def store_config(self, env_cfg: dict | object, train_cfg: dict) -> None:
        """Called once at the start of training."""

    def save_model(self, model_path: str, it: int) -> None:
        """Upload a checkpoint."""

    def save_file(self, path: str) -> None:
        """Upload a file."""

    def save_video(self, video: pathlib.Path, it: int) -> None:
        """Upload a video."""

    def stop(self) -> None:
        """Close the run."""

    def abort(self) -> None:
        """Close the run after an interruption (defaults to :meth:`stop`)."""
        self.stop()


class CsvLogWriter(LogWriter):
    """One CSV row per iteration (``metrics.csv``) plus ``config.json`` in ``log_dir`` (no external service).

    Columns are ``iteration``, ``wall_s`` (seconds since the writer was made) and then every tag in order of first
    appearance; a tag that starts late (``Train/mean_reward`` appears once the first episode ends) gets its own column
    and empty cells before. The file is rewritten whenever an iteration completes, so an interrupted run still leaves
    a valid CSV. Time-indexed duplicates (``*/time`` tags, stepped by seconds rather than iterations, which a logger
    emits for writers of other kinds) are skipped: ``wall_s`` carries the time."""

    def __init__(self, log_dir: str, filename: str = "metrics.csv", **kwargs) -> None:
        self.log_dir = log_dir
        os.makedirs(log_dir, exist_ok=True)
        self.path = os.path.join(log_dir, filename)
        self._t0 = time.time()
        self._rows: dict[int, dict[str, float]] = {}
        self._columns: list[str] = []
        self._step: int | None = None

    def add_scalar(self, tag: str, scalar_value: float, global_step: int) -> None:
        if tag.endswith("/time"):
            return
        if self._step is not None and global_step != self._step:
            self._flush()
        self._step = global_step
        row = self._rows.setdefault(global_step, {"iteration": global_step,
                                                  "wall_s": round(time.time() - self._t0, 3)})
        row[tag] = float(scalar_value)
        if tag not in self._columns:
            self._columns.append(tag)

    def _flush(self) -> None:
        if not self._rows:
            return
        with open(self.path, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=["iteration", "wall_s", *self._columns], restval="")
            w.writeheader()
            for step in sorted(self._rows):
                w.writerow(self._rows[step])

    def store_config(self, env_cfg: dict | object, train_cfg: dict) -> None:
        def default(o):
            return repr(o)

        with open(os.path.join(self.log_dir, "config.json"), "w") as f:
            json.dump({"env_cfg": env_cfg if isinstance(env_cfg, dict) else repr(env_cfg), "train_cfg": train_cfg}, f,
                      default=default, indent=2)

    def stop(self) -> None:
        self._flush()
