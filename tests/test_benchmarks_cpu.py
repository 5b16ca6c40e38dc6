"""The algorithm-cost matrix (null environment, both implementations) and the bridge benchmark, on tiny sizes."""

import pytest
import torch


@pytest.mark.parametrize("impl", ["b200", "upstream"])
def test_bench_matrix_reports_every_phase(ref, impl):
    from tt_rsl_rl_b200.runners.bench_matrix import matrix

    (res,) = list(matrix(impl, "cpu", [64], [[32, 32]], steps=4, iters=1, warmup=1, mini_batches=2, epochs=1))
    for k in ("act_ms", "env_ms", "process_ms", "returns_ms", "update_ms", "total_ms"):
        assert res[k] >= 0.0
    assert res["total_ms"] >= res["update_ms"] and res["env_steps_per_s"] > 0
    assert res["impl"] == impl and res["num_envs"] == 64


def test_null_env_is_constant():
    from tt_rsl_rl_b200.env.null import NullVecEnv

    env = NullVecEnv(8, {"policy": 3, "critic": 5}, 2)
    o0 = env.get_observations()
    o1, r, d, e = env.step(torch.zeros(8, 2))
    assert o1["critic"].shape == (8, 5) and torch.equal(o0["policy"], o1["policy"])
    assert not bool(d.any()) and not bool(e["time_outs"].any())


@pytest.mark.parametrize("transport", ["zmq-tcp", "zmq-pickle", "raw-tcp"])
def test_bridge_bench_round_trips(transport):
    from tt_rsl_rl_b200.env.bench_bridge import measure, step_bytes

    res = measure(transport, 64, steps=5, warmup=2)
    assert res["ms_per_step"] > 0 and res["bytes_per_step"] == sum(step_bytes(64, {"policy": 36, "privileged": 48}, 12))
