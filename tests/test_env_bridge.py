"""Remote environment bridge over ZeroMQ (loopback): equality with the local environment, error replies, timeouts,
and a runner learning through the bridge."""

import pytest
import torch

zmq = pytest.importorskip("zmq")


def _server(env):
    from tt_rsl_rl_b200.env import EnvServer

    srv = EnvServer(env, "tcp://127.0.0.1:*")
    srv.serve_in_thread()
    return srv


def test_bridge_steps_equal_the_local_environment():
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv, RemoteVecEnv

    local = LinearGaussianVecEnv(64, obs_dim=10, num_actions=3, privileged_dim=2, seed=4, reset_prob=0.1)
    served = LinearGaussianVecEnv(64, obs_dim=10, num_actions=3, privileged_dim=2, seed=4, reset_prob=0.1)
    srv = _server(served)
    remote = RemoteVecEnv(srv.address, timeout_ms=5000)
    assert (remote.num_envs, remote.num_actions) == (64, 3)
    assert remote.groups == {"policy": [10], "critic": [12]}
    torch.testing.assert_close(remote.get_observations()["critic"], local.get_observations()["critic"])
    torch.manual_seed(0)
    for _ in range(5):
        a = torch.randn(64, 3)
        torch.manual_seed(1)  # the environments draw their noise from the global generator
        o1, r1, d1, e1 = local.step(a)
        torch.manual_seed(1)
        o2, r2, d2, e2 = remote.step(a)
        torch.testing.assert_close(o2["policy"], o1["policy"])
        torch.testing.assert_close(r2, r1)
        torch.testing.assert_close(d2, d1.float())
        torch.testing.assert_close(remote.episode_length_buf, local.episode_length_buf)
        if "time_outs" in e1:
            torch.testing.assert_close(e2["time_outs"], e1["time_outs"].float())
    remote.close()


def test_bridge_server_survives_handler_errors():
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv, RemoteEnvError, RemoteVecEnv

    srv = _server(LinearGaussianVecEnv(8, obs_dim=4, num_actions=2))
    remote = RemoteVecEnv(srv.address, timeout_ms=5000)
    with pytest.raises(RemoteEnvError, match="actions must have shape"):
        remote.step(torch.zeros(8, 5))
    obs, rew, dones, _ = remote.step(torch.zeros(8, 2))  # still serving
    assert rew.shape == (8,) and srv.errors == 1
    remote.close()


def test_bridge_client_times_out_instead_of_hanging():
    import time

    from tt_rsl_rl_b200.env import LinearGaussianVecEnv, RemoteEnvTimeoutError, RemoteVecEnv

    srv = _server(LinearGaussianVecEnv(8, obs_dim=4, num_actions=2))
    remote = RemoteVecEnv(srv.address, timeout_ms=3000)
    srv.stop()  # the server goes away: no reply to the next request
    time.sleep(0.3)
    remote.timeout_ms = 500
    remote.sock.close(0)
    remote._connect()
    t0 = time.monotonic()
    with pytest.raises(RemoteEnvTimeoutError):
        remote.step(torch.zeros(8, 2))
    assert time.monotonic() - t0 < 3.0


def test_runner_learns_through_the_bridge(tmp_path):
    import copy

    from helpers import ppo_cfg

    from tt_rsl_rl_b200.env import LinearGaussianVecEnv, RemoteVecEnv
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    srv = _server(LinearGaussianVecEnv(32, obs_dim=6, num_actions=2, privileged_dim=1))
    remote = RemoteVecEnv(srv.address, timeout_ms=5000)
    runner = OnPolicyRunner(remote, copy.deepcopy(ppo_cfg(T=4)), log_dir=None, device="cpu")
    runner.learn(2)
    assert runner.current_learning_iteration == 1
    remote.close()


def test_training_through_the_bridge_equals_local_training():
    """Loopback equality: the same seeds give bit-identical parameters whether the environment is local or behind the
    bridge (the transport moves raw float32 bytes, nothing is re-encoded)."""
    import copy

    from helpers import ppo_cfg

    from tt_rsl_rl_b200.env import LinearGaussianVecEnv, RemoteVecEnv
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    def make_env():
        return LinearGaussianVecEnv(32, obs_dim=6, num_actions=2, privileged_dim=1, seed=4)

    def train(env):
        torch.manual_seed(9)
        runner = OnPolicyRunner(env, copy.deepcopy(ppo_cfg(T=4)), log_dir=None, device="cpu")
        runner.learn(3)
        return [p.detach().clone() for p in runner.alg.actor.parameters()]

    local = train(make_env())
    srv = _server(make_env())
    remote = RemoteVecEnv(srv.address, timeout_ms=5000)
    try:
        bridged = train(remote)
    finally:
        remote.close()
    for a, b in zip(local, bridged):
        assert torch.equal(a, b)


def test_agent_cfg_conversion_and_loading(tmp_path):
    import json

    import yaml

    from helpers import ppo_cfg

    from tt_rsl_rl_b200.env import b200_agent_cfg, load_agent_cfg

    host = ppo_cfg()
    host["class_name"] = "OnPolicyRunner"
    host["algorithm"]["class_name"] = "rsl_rl.algorithms:PPO"
    host["actor"]["class_name"] = "rsl_rl.models.MLPModel"
    host["actor"]["distribution_cfg"]["class_name"] = "rsl_rl.modules:GaussianDistribution"
    before = json.dumps(host, sort_keys=True)
    cfg = b200_agent_cfg(host, device="cuda:1", graphs=False, csv_log=True, extra_b200_cfg={"section_timing": True})
    assert json.dumps(host, sort_keys=True) == before  # the argument is not modified
    assert cfg["algorithm"]["class_name"] == "PPO" and cfg["actor"]["class_name"] == "MLPModel"
    assert cfg["actor"]["distribution_cfg"]["class_name"] == "GaussianDistribution"
    assert cfg["algorithm"]["b200_cfg"] == {"engine": "auto", "graphs": False, "section_timing": True}
    assert cfg["device"] == "cuda:1" and cfg["logger"]["class_name"].endswith(":CsvLogWriter")
    assert cfg["actor"]["hidden_dims"] == host["actor"]["hidden_dims"] and cfg["obs_groups"] == host["obs_groups"]
    with pytest.raises(NotImplementedError):
        b200_agent_cfg({**host, "class_name": "OffPolicyRunner"})
    with pytest.raises(NotImplementedError):
        b200_agent_cfg({**host, "algorithm": {"class_name": "SAC"}})
    with pytest.raises(ValueError, match="critic"):
        b200_agent_cfg({k: v for k, v in host.items() if k != "critic"})
    dist = {"class_name": "DistillationRunner", "obs_groups": {}, "student": {}, "teacher": {},
            "algorithm": {"class_name": "rsl_rl.algorithms:Distillation"}}
    assert b200_agent_cfg(dist)["algorithm"]["class_name"] == "Distillation"
    # JSON and YAML (Isaac Lab dumps tuples with a Python tag)
    (tmp_path / "agent.json").write_text(json.dumps(host))
    assert load_agent_cfg(tmp_path / "agent.json") == host
    (tmp_path / "agent.yaml").write_text(yaml.dump({**host, "clip_actions": (1.0, 2.0)}))
    loaded = load_agent_cfg(tmp_path / "agent.yaml")
    assert loaded["clip_actions"] == (1.0, 2.0) and loaded["actor"] == host["actor"]
    (tmp_path / "bad.json").write_text("[1, 2]")
    with pytest.raises(ValueError):
        load_agent_cfg(tmp_path / "bad.json")


def test_server_hands_its_agent_cfg_to_the_learner():
    import copy

    from helpers import ppo_cfg

    from tt_rsl_rl_b200.env import EnvServer, LinearGaussianVecEnv, RemoteVecEnv, b200_agent_cfg
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    host_cfg = ppo_cfg(T=4)
    srv = EnvServer(LinearGaussianVecEnv(16, obs_dim=6, num_actions=2, privileged_dim=1), "tcp://127.0.0.1:*",
                    agent_cfg=host_cfg)
    srv.serve_in_thread()
    remote = RemoteVecEnv(srv.address, timeout_ms=5000)
    try:
        assert remote.agent_cfg == host_cfg
        cfg = b200_agent_cfg(remote.agent_cfg, device="cpu")
        runner = OnPolicyRunner(remote, copy.deepcopy(cfg), log_dir=None, device=cfg["device"])
        runner.learn(1)
    finally:
        remote.close()


def test_episode_lengths_reset_protocol_and_stats():
    import copy

    from helpers import ppo_cfg

    from tt_rsl_rl_b200.env import EnvServer, LinearGaussianVecEnv, RemoteEnvError, RemoteVecEnv
    from tt_rsl_rl_b200.env import bridge as B
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    class ResettableEnv(LinearGaussianVecEnv):
        resets = 0

        def reset(self):
            ResettableEnv.resets += 1
            self.episode_length_buf.zero_()
            return self.get_observations(), {"log": {"resets": torch.tensor(float(ResettableEnv.resets))}}

    local = ResettableEnv(16, obs_dim=6, num_actions=2, privileged_dim=1, episode_length=50)
    srv = EnvServer(local, "tcp://127.0.0.1:*")
    srv.serve_in_thread()
    remote = RemoteVecEnv(srv.address, timeout_ms=5000)
    try:
        assert remote.has_reset
        # the runner's random start lengths reach the simulator
        runner = OnPolicyRunner(remote, copy.deepcopy(ppo_cfg(T=4)), log_dir=None, device="cpu")
        runner.learn(1, init_at_random_ep_len=True)
        assert int(local.episode_length_buf.max()) > 4 and torch.equal(remote.episode_length_buf,
                                                                      local.episode_length_buf)
        obs, extras = remote.reset()
        assert ResettableEnv.resets == 1 and extras["log"]["resets"] == 1.0
        assert int(remote.episode_length_buf.sum()) == 0 and obs["policy"].shape == (16, 6)
        s = remote.stats.summary()
        assert s["step"]["calls"] == 4 and s["set_episode_length_buf"]["calls"] == 1 and s["reset"]["calls"] == 1
        assert s["received_bytes"] > s["sent_bytes"] > 0
    finally:
        remote.close()
    # a server of another protocol version is refused
    srv2 = EnvServer(LinearGaussianVecEnv(4, obs_dim=3, num_actions=1), "tcp://127.0.0.1:*")
    inner = srv2._handle

    def older_server(header, tensors):
        out = inner(header, tensors)
        if header.get("op") == "info":
            out[0]["protocol"] = B.PROTOCOL_VERSION - 1
        return out

    srv2._handle = older_server
    srv2.serve_in_thread()
    try:
        with pytest.raises(RemoteEnvError, match="protocol"):
            RemoteVecEnv(srv2.address, timeout_ms=5000)
    finally:
        srv2.stop()


def test_command_line_serve_and_train(tmp_path):
    """The environment host serves a test environment with its run spec; the learner trains against it with the
    configuration the server sent, writes metrics and checkpoints, and closing the client stops the server."""
    import socket
    import subprocess
    import sys

    from tt_rsl_rl_b200.env import bridge

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = subprocess.Popen([sys.executable, "-m", "tt_rsl_rl_b200.env.bridge", "serve", "--local-env", "cartpole",
                               "--num-envs", "32", "--address", f"tcp://127.0.0.1:{port}"],
                              stdout=subprocess.PIPE, text=True)
    try:
        assert "serving" in server.stdout.readline()
        rc = bridge.main(["train", "--address", f"tcp://127.0.0.1:{port}", "--iterations", "2",
                          "--log-dir", str(tmp_path), "--device", "cpu", "--timeout-ms", "30000"])
        assert rc == 0
        assert server.wait(timeout=30) == 0
    finally:
        if server.poll() is None:
            server.kill()
            server.wait()
    import csv

    rows = list(csv.DictReader(open(tmp_path / "metrics.csv")))
    assert [r["iteration"] for r in rows] == ["0", "1"] and (tmp_path / "model_1.pt").exists()
