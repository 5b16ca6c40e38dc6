"""The fused linear-Gaussian environment step against its PyTorch-op specification (same process noise supplied by
the caller; resets statistically, as their random streams differ)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _pair(N=4096, reset_prob=0.0, episode_length=10**6, privileged_dim=3):
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv

    kw = dict(obs_dim=96, num_actions=29, privileged_dim=privileged_dim, device="cuda", seed=7, host_noise=True,
              reset_prob=reset_prob, episode_length=episode_length)
    return LinearGaussianVecEnv(N, fused=False, **kw), LinearGaussianVecEnv(N, fused=True, **kw)


def test_fused_step_matches_specification_without_resets():
    ref, fused = _pair()
    assert fused.fused and not ref.fused
    for _ in range(5):
        a = torch.randn(4096, 29, device="cuda")
        o1, r1, d1, e1 = ref.step(a)
        o2, r2, d2, e2 = fused.step(a)
        torch.testing.assert_close(o2["policy"], o1["policy"], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(o2["critic"], o1["critic"], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(r2, r1, rtol=1e-5, atol=1e-4)
        assert d2.sum() == 0 and torch.equal(fused.episode_length_buf, ref.episode_length_buf)


def test_fused_resets_and_time_outs():
    _, env = _pair(N=65536, reset_prob=0.05, episode_length=7)
    terms = 0
    for t in range(1, 15):
        _, _, d, e = env.step(torch.zeros(65536, 29, device="cuda"))
        to = e["time_outs"]
        terms += int((d - to).sum())
        if t % 7 == 0:  # every environment that survived 7 steps times out now
            assert int(to.sum()) > 0
    rate = terms / (14 * 65536)
    assert 0.04 < rate < 0.06, rate
    # reset states are standard normal; the privileged length feature is 0 for a fresh episode
    s = env.state[env.episode_length_buf == 0]
    assert abs(float(s.mean())) < 0.02 and abs(float(s.std()) - 1.0) < 0.02
    crit = env.get_observations()["critic"]
    fresh = env.episode_length_buf == 0
    assert torch.all(crit[fresh, 96 + 2] == 0)


def test_runner_with_fused_env_captured_rollout():
    import copy

    from tt_rsl_rl_b200.env import humanoid_like
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    cfg = {
        "num_steps_per_env": 8, "save_interval": 1000, "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "algorithm": {"class_name": "PPO", "num_learning_epochs": 1, "num_mini_batches": 2,
                      "b200_cfg": {"engine": "cuda"}},
        "actor": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True,
                  "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True},
    }
    env = humanoid_like(1024, device="cuda", seed=1)
    assert env.fused and env.graph_capturable
    runner = OnPolicyRunner(env, copy.deepcopy(cfg), log_dir=None, device="cuda")
    runner.learn(3)  # eager rollout, then a captured one, then a replay
    assert torch.isfinite(runner.alg.engine.flat).all()
    assert int(env._env_counter.item()) == 3 * 8


def test_inplace_pytorch_step_is_captured_with_the_rollout():
    """The benchmark's environment on this framework's arm: the PyTorch-op step rewriting its observations in place,
    captured with the rollout as one CUDA graph (the torch generator advances on every replay)."""
    import copy

    from tt_rsl_rl_b200.env import humanoid_like
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    cfg = {
        "num_steps_per_env": 8, "save_interval": 1000, "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
        "algorithm": {"class_name": "PPO", "num_learning_epochs": 1, "num_mini_batches": 2,
                      "b200_cfg": {"engine": "cuda"}},
        "actor": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True,
                  "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
        "critic": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True},
    }
    env = humanoid_like(1024, device="cuda", seed=1, fused=False, inplace_obs=True, host_noise=True,
                        rollout_steps=8)
    assert not env.fused and env.graph_capturable
    obs0 = env.get_observations()["policy"]
    runner = OnPolicyRunner(env, copy.deepcopy(cfg), log_dir=None, device="cuda")
    runner.learn(3)  # eager rollout, then a captured one, then a replay
    torch.cuda.synchronize()
    assert runner.alg.engine._rollout_graph is not None
    assert env.get_observations()["policy"].data_ptr() == obs0.data_ptr()
    assert torch.isfinite(runner.alg.engine.flat).all()
    s1 = env.state.clone()
    runner.learn(1)
    assert not torch.equal(env.state, s1)  # replays keep stepping the environment


def test_prefetched_host_noise_equals_inline_copies():
    from tt_rsl_rl_b200.env import humanoid_like

    def run(rollout_steps):
        torch.manual_seed(3)
        env = humanoid_like(2048, device="cuda", seed=2, fused=False, host_noise=True, rollout_steps=rollout_steps)
        g = torch.Generator(device="cuda").manual_seed(5)
        out = []
        for _ in range(9):  # crosses two prefetch windows of 4 steps
            a = torch.randn(2048, 29, device="cuda", generator=g)
            o, r, d, _ = env.step(a)
            out.append((o["critic"].clone(), r.clone(), d.clone()))
        torch.cuda.synchronize()
        return out

    for (o1, r1, d1), (o2, r2, d2) in zip(run(None), run(4)):
        assert torch.equal(o1, o2) and torch.equal(r1, r2) and torch.equal(d1, d2)
