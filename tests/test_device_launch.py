"""Device guard (checks, per-GPU lock, close hooks) with fake system calls, and the job launcher (locks, records,
time limit with interrupt then kill, restart of a failed job that resumes from its newest checkpoint) with host-only
child processes."""

import json
import os
import subprocess
import sys
import textwrap
import time

import pytest

from tt_rsl_rl_b200 import device as dev
from tt_rsl_rl_b200 import launch


def _deps(tmp_path, **kw):
    calls = {"set_device": [], "sync": []}
    base = dict(environ={"TT_RSL_RL_LOCK_DIR": str(tmp_path / "locks")}, cuda_available=lambda: True,
                device_count=lambda: 2, capability=lambda i: (10, 0), mem_get_info=lambda i: (100 << 30, 180 << 30),
                load_extension=lambda: object(), set_device=lambda i: calls["set_device"].append(i),
                synchronize=lambda i: calls["sync"].append(i))
    base.update(kw)
    return dev.Deps(**base), calls


@pytest.fixture(autouse=True)
def _no_open_session():
    yield
    s = dev.active_session()
    if s is not None:
        s.close()


def test_guard_opens_locks_and_closes_in_order(tmp_path):
    deps, calls = _deps(tmp_path)
    order = []
    with dev.open_gpu(1, deps=deps) as s:
        assert s.device == "cuda:1" and calls["set_device"] == [1] and s.lock_held
        assert dev.GpuLock.holder(dev.lock_path(1, str(tmp_path / "locks"))) == str(os.getpid())
        assert dev.acquire_gpu(deps=deps) is s  # the owner keeps the open session
        with pytest.raises(dev.DeviceGuardError, match="cannot switch"):
            dev.acquire_gpu(0, deps=deps)
        with pytest.raises(dev.DeviceGuardError, match="already open"):
            dev.open_gpu(1, deps=deps)
        s.add_close_hook(lambda: order.append("first"))
        s.add_close_hook(lambda: order.append("second"))
    assert order == ["second", "first"] and calls["sync"] == [1] and not s.lock_held
    s.close()  # idempotent
    assert order == ["second", "first"] and dev.active_session() is None


@pytest.mark.parametrize("case,kw,match", [
    ("no cuda", dict(cuda_available=lambda: False), "no CUDA device"),
    ("index", dict(device_count=lambda: 1), "out of range"),
    ("arch", dict(capability=lambda i: (9, 0)), "compute capability 9.0"),
    ("memory", dict(mem_get_info=lambda i: (1 << 30, 180 << 30)), "GiB required"),
    ("extension", dict(load_extension=lambda: (_ for _ in ()).throw(ImportError("no _C"))), "does not load"),
])
def test_guard_refusals_release_the_lock(tmp_path, case, kw, match):
    deps, calls = _deps(tmp_path, **kw)
    with pytest.raises(dev.DeviceGuardError, match=match):
        dev.open_gpu(1, deps=deps, min_free_bytes=8 << 30)
    assert calls["set_device"] == [] and dev.active_session() is None
    # whatever failed, the GPU's lock is free again
    lk = dev.GpuLock(dev.lock_path(1, str(tmp_path / "locks")))
    lk.acquire()
    lk.release()


def test_guard_refuses_a_gpu_locked_by_another_process(tmp_path):
    locks = tmp_path / "locks"
    holder = subprocess.Popen([sys.executable, "-c", textwrap.dedent(f"""
        import sys, time
        sys.path.insert(0, {os.getcwd()!r})
        from tt_rsl_rl_b200.device import GpuLock, lock_path
        GpuLock(lock_path(0, {str(locks)!r})).acquire()
        print("held", flush=True)
        time.sleep(60)
    """)], stdout=subprocess.PIPE, text=True)
    try:
        assert holder.stdout.readline().strip() == "held"
        deps, _ = _deps(tmp_path)
        with pytest.raises(dev.DeviceGuardError, match=f"held by process {holder.pid}"):
            dev.open_gpu(0, deps=deps)
        # the launcher of this job holds it: no second lock is taken
        deps2, _ = _deps(tmp_path, environ={"TT_RSL_RL_LOCK_DIR": str(locks), dev.LOCKS_HELD_ENV: "0"})
        with dev.open_gpu(0, deps=deps2) as s:
            assert not s.lock_held
    finally:
        holder.kill()
        holder.wait()


def test_physical_index_follows_visible_devices():
    assert dev.physical_index(1, {"CUDA_VISIBLE_DEVICES": "4,6"}) == 6
    assert dev.physical_index(0, {}) == 0
    assert dev.physical_index(0, {"CUDA_VISIBLE_DEVICES": "GPU-abc"}) == "GPU-abc"


# ---- launcher -----------------------------------------------------------------------------------------------------------
def _script(tmp_path, body):
    p = tmp_path / "job.py"
    p.write_text(textwrap.dedent(body))
    return str(p)


def test_launch_runs_ranks_through_torchrun(tmp_path):
    out = tmp_path / "out"
    out.mkdir()
    script = _script(tmp_path, f"""
        import os
        with open(os.path.join({str(out)!r}, os.environ["RANK"]), "w") as f:
            f.write(os.environ["WORLD_SIZE"] + " " + os.environ["MASTER_ADDR"])
    """)
    rc = launch.run_job([script], gpus=[], nproc=2, timeout=120, run_dir=str(tmp_path / "jobs"),
                        lock_dir=str(tmp_path / "locks"))
    assert rc == 0
    assert sorted(os.listdir(out)) == ["0", "1"]
    assert (out / "1").read_text() == "2 127.0.0.1"
    assert launch.list_jobs(str(tmp_path / "jobs")) == []  # the record is gone after the job


def test_launch_timeout_interrupts_then_kills(tmp_path):
    marker = tmp_path / "interrupted"
    script = _script(tmp_path, f"""
        import time
        try:
            time.sleep(60)
        except KeyboardInterrupt:
            open({str(marker)!r}, "w").write("yes")
            time.sleep(60)  # ignores the interrupt's intent: the launcher must kill it
    """)
    t0 = time.monotonic()
    rc = launch.run_job([script], gpus=[], timeout=1.0, grace=1.0, torchrun=False, run_dir=str(tmp_path / "jobs"),
                        lock_dir=str(tmp_path / "locks"))
    assert rc == launch.EXIT_TIMEOUT and marker.read_text() == "yes"
    assert time.monotonic() - t0 < 30


def test_launch_refuses_a_locked_gpu_and_records_running_jobs(tmp_path):
    locks, jobs = str(tmp_path / "locks"), str(tmp_path / "jobs")
    lk = dev.GpuLock(dev.lock_path(3, locks))
    lk.acquire()
    try:
        rc = launch.run_job(["-c", "pass"], gpus=[3], torchrun=False, run_dir=jobs, lock_dir=locks)
        assert rc == launch.EXIT_REFUSED
    finally:
        lk.release()
    script = _script(tmp_path, """
        import os, time
        assert os.environ["CUDA_VISIBLE_DEVICES"] == "3" and os.environ["TT_RSL_RL_GPU_LOCKS_HELD"] == "3"
        time.sleep(60)
    """)
    proc = subprocess.Popen([sys.executable, "-m", "tt_rsl_rl_b200.launch", "--gpus", "3", "--no-torchrun",
                             "--tag", "sleeper", "--grace", "2", "--run-dir", jobs, "--lock-dir", locks, "--", script],
                            cwd=os.getcwd())
    try:
        for _ in range(200):
            recs = launch.list_jobs(jobs)
            if recs:
                break
            time.sleep(0.05)
        assert len(recs) == 1 and recs[0]["tag"] == "sleeper" and recs[0]["gpus"] == [3]
        assert launch.lock_holders(locks) == {"gpu3.lock": str(proc.pid)}
        assert launch.stop_mine("sleeper", jobs) == [recs[0]["pgid"]]
        assert proc.wait(timeout=30) != 0
    finally:
        if proc.poll() is None:
            proc.kill()
            proc.wait()
    assert launch.list_jobs(jobs) == []
    out = subprocess.run([sys.executable, "-m", "tt_rsl_rl_b200.launch", "--list", "--run-dir", jobs,
                          "--lock-dir", locks], capture_output=True, text=True, check=True)
    assert json.loads(out.stdout)["jobs"] == []


def test_failed_job_is_restarted_and_resumes_from_its_newest_checkpoint(tmp_path):
    """Attempt 0 crashes in its third iteration (after checkpoints of iterations 0 and 1); attempt 1 resumes from the
    newest one and finishes the run."""
    logs = tmp_path / "run"
    script = _script(tmp_path, f"""
        import copy, json, os, sys
        sys.path.insert(0, {os.path.join(os.getcwd(), "tests")!r})
        sys.path.insert(0, {os.getcwd()!r})
        import torch
        from helpers import ppo_cfg, small_env
        from tt_rsl_rl_b200.runners import OnPolicyRunner

        attempt = int(os.environ["TT_RSL_RL_ATTEMPT"])
        env = small_env(8)
        if attempt == 0:
            step = env.step
            calls = [0]

            def failing(actions):
                calls[0] += 1
                if calls[0] > 2 * 4 + 1:  # inside the third iteration (4 steps each)
                    raise RuntimeError("simulator crashed")
                return step(actions)

            env.step = failing
        cfg = ppo_cfg(T=4)
        cfg["save_interval"] = 1
        cfg["logger"] = {{"class_name": "CsvLogWriter"}}
        runner = OnPolicyRunner(env, copy.deepcopy(cfg), log_dir={str(logs)!r}, device="cpu")
        resumed = runner.resume_latest()
        with open(os.path.join({str(tmp_path)!r}, f"attempt{{attempt}}.json"), "w") as f:
            json.dump({{"resumed": resumed, "start": runner.current_learning_iteration}}, f)
        runner.learn(4 - runner.current_learning_iteration)
    """)
    rc = launch.run_job([script], gpus=[], torchrun=False, retries=2, run_dir=str(tmp_path / "jobs"),
                        lock_dir=str(tmp_path / "locks"), timeout=300)
    assert rc == 0
    a0 = json.loads((tmp_path / "attempt0.json").read_text())
    a1 = json.loads((tmp_path / "attempt1.json").read_text())
    assert a0 == {"resumed": None, "start": 0}
    assert a1["resumed"].endswith("model_1.pt") and a1["start"] == 1
    assert not (tmp_path / "attempt2.json").exists()
    from tt_rsl_rl_b200.runners import latest_checkpoint

    assert latest_checkpoint(str(logs)).endswith("model_3.pt")
    assert latest_checkpoint(str(tmp_path / "missing")) is None
