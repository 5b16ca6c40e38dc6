"""The device guard and the job launcher on a real B200 (their host logic is tested with fakes in
tests/test_device_launch.py)."""

import copy
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(guard):
    return {
        "num_steps_per_env": 4, "save_interval": 1000, "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "algorithm": {"class_name": "PPO", "num_learning_epochs": 1, "num_mini_batches": 2,
                      "b200_cfg": {"engine": "cuda"}},
        "actor": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True,
                  "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True},
        "device_guard": guard,
    }


def test_runner_with_device_guard_opens_and_locks_the_gpu(tmp_path):
    from tt_rsl_rl_b200.device import active_session, lock_path, physical_index
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    env = LinearGaussianVecEnv(256, obs_dim=24, num_actions=6, privileged_dim=3, device="cuda:0")
    runner = OnPolicyRunner(env, copy.deepcopy(_cfg({"lock_dir": str(tmp_path)})), log_dir=None, device="cuda:0")
    session = runner.gpu_session
    assert session is not None and active_session() is session
    assert os.path.exists(lock_path(physical_index(0, os.environ), str(tmp_path)))
    runner.learn(1)
    assert torch.isfinite(runner.alg.engine.flat).all()
    session.close()
    session.close()  # idempotent


def test_launcher_runs_a_gpu_job_under_its_lock(tmp_path):
    script = os.path.join(ROOT, "examples", "tracking12", "train.py")
    cmd = [sys.executable, "-m", "tt_rsl_rl_b200.launch", "--gpus", "0", "--timeout", "300", "--no-torchrun",
           "--tag", "gpu-test", "--run-dir", str(tmp_path / "runs"), "--lock-dir", str(tmp_path / "locks"), "--",
           script, "--device", "cuda:0", "--envs", "256", "--iterations", "2", "--log-dir", str(tmp_path / "log"),
           "--engine", "cuda"]
    out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
    assert any(f.startswith("model_") for f in os.listdir(tmp_path / "log"))
