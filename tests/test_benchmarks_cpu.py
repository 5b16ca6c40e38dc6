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


def test_op_profiler_times_launching_entry_points(monkeypatch):
    from tt_rsl_rl_b200 import ops

    class FakeExt:
        def gae(self, x):
            return x + 1

        def gemm(self, x):
            return x * 2

        def plan_sizes(self):
            return "host helper"

    class FakeEvent:
        clock = [0.0]

        def record(self):
            FakeEvent.clock[0] += 0.5
            self.t = FakeEvent.clock[0]

        def elapsed_time(self, end):
            return end.t - self.t

    monkeypatch.setattr(ops, "_EXT", FakeExt())
    capturing = {"on": False}
    with ops.count_launches() as cnt, ops.profile_ops(FakeEvent, lambda: None, lambda: capturing["on"]) as prof:
        assert ops.ext().gae(1) == 2 and ops.ext().gae(2) == 3 and ops.ext().gemm(3) == 6
        assert ops.ext().plan_sizes() == "host helper"  # not a launching entry point: neither counted nor timed
        capturing["on"] = True
        ops.ext().gemm(1)  # inside a graph capture: counted, not timed
    assert cnt.n == 4
    assert prof.stats == {"gae": [2, 1.0], "gemm": [1, 0.5]}
    rows = prof.table()
    assert rows[0]["op"] == "gae" and rows[0]["mean_us"] == 500.0 and abs(sum(r["share"] for r in rows) - 1) < 1e-6
    assert ops._PROFILER is None and ops.ext() is ops._EXT  # instrumentation ends with the block
    with pytest.raises(RuntimeError):
        with ops.profile_ops(FakeEvent, lambda: None, lambda: False), ops.profile_ops(FakeEvent):
            pass
    assert ops._PROFILER is None


def test_bridge_bench_runs_the_reference_bridge(ref):
    from tt_rsl_rl_b200.env.bench_bridge import measure

    res = measure("reference-zmq-tcp", 64, steps=5, warmup=2)
    assert res["ms_per_step"] > 0 and res["bytes_per_step"] > 64 * 4 * (36 + 48)
