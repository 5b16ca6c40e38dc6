"""Seeded batched test environments and a learning check (golden-curve style: the trained policy must clearly beat the
initial one on a fixed evaluation)."""

import copy

import torch


def test_seeded_and_shaped():
    from tt_rsl_rl_b200.env.classic import (BatchedCartPole, BatchedCartPoleImage, BatchedCartPolePO, BatchedPendulum,
                                            Tracking12)

    for cls, dims in ((BatchedCartPole, {"policy": 4}), (BatchedCartPolePO, {"policy": 2}),
                      (BatchedCartPoleImage, {"policy": 2, "image": 1}),
                      (BatchedPendulum, {"policy": 3}), (Tracking12, {"policy": 36, "privileged": 48})):
        a, b, c = cls(16, seed=3), cls(16, seed=3), cls(16, seed=4)
        obs = a.get_observations()
        assert {g: obs[g].shape[1] for g in obs.keys()} == dims
        act = torch.randn(16, cls.num_actions)
        oa, ra, da, ea = a.step(act)
        ob, rb, db, eb = b.step(act)
        oc = c.step(act)[0]
        for g in dims:
            torch.testing.assert_close(oa[g], ob[g])
        assert not all(torch.equal(oa[g], oc[g]) for g in dims)
        assert ra.shape == (16,) and da.shape == (16,) and "time_outs" in ea and ea["log"]


def test_cartpole_falls_without_control_and_times_out():
    from tt_rsl_rl_b200.env.classic import BatchedCartPole, BatchedPendulum

    env = BatchedCartPole(64, seed=0)
    done_any = torch.zeros(64, dtype=torch.bool)
    for _ in range(300):
        _, _, d, e = env.step(torch.zeros(64, 1))
        done_any |= d.bool() & (e["time_outs"] == 0)
    assert done_any.all()  # every pole falls (terminations, not time-outs)
    pend = BatchedPendulum(8, seed=0)
    n_timeouts = 0
    for _ in range(200):
        _, _, d, e = pend.step(torch.zeros(8, 1))
        n_timeouts += int(e["time_outs"].sum())
    assert n_timeouts == 8


def _evaluate(runner, env_cls, steps=200):
    env = env_cls(128, seed=123)
    policy = runner.get_inference_policy()
    obs = env.get_observations()
    alive = torch.ones(128)
    survived = torch.zeros(128)
    with torch.no_grad():
        for _ in range(steps):
            obs, _, d, _ = env.step(policy(obs))
            survived += alive
            alive = alive * (1 - d)
    return float(survived.mean())


def test_ppo_learns_cartpole():
    from helpers import ppo_cfg

    from tt_rsl_rl_b200.env.classic import BatchedCartPole
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    torch.manual_seed(0)
    cfg = copy.deepcopy(ppo_cfg(hidden=(64, 64), T=32, epochs=5, mbs=4, critic_group="policy"))
    cfg["actor"]["distribution_cfg"]["init_std"] = 0.5
    runner = OnPolicyRunner(BatchedCartPole(256, seed=1), cfg, log_dir=None, device="cpu")
    before = _evaluate(runner, BatchedCartPole)
    runner.learn(25)
    after = _evaluate(runner, BatchedCartPole)
    assert after > 2.0 * before and after > 60, (before, after)
