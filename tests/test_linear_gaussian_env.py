"""Observation-buffer modes of the synthetic linear-Gaussian environment (host only)."""

import torch

from tt_rsl_rl_b200.env import LinearGaussianVecEnv


def _run(inplace_obs):
    torch.manual_seed(0)
    env = LinearGaussianVecEnv(64, obs_dim=10, num_actions=3, privileged_dim=3, seed=4, reset_prob=0.2,
                               episode_length=5, inplace_obs=inplace_obs)
    g = torch.Generator().manual_seed(1)
    out, ptrs, kept = [], set(), True
    prev = env.get_observations()
    for _ in range(12):
        before = prev["critic"].clone()
        obs, rew, done, extras = env.step(torch.randn(64, 3, generator=g))
        if not inplace_obs:
            kept &= torch.equal(prev["critic"], before)  # the observations acted on stay intact
        prev = obs
        ptrs.add(obs["policy"].data_ptr())
        out.append((obs["critic"].clone(), rew.clone(), done.clone(), extras["time_outs"].clone()))
    return env, out, ptrs, kept


def test_inplace_and_alternating_buffers_give_the_same_trajectory():
    env_a, out_a, ptrs_a, kept = _run(False)
    env_b, out_b, ptrs_b, _ = _run(True)
    assert kept and len(ptrs_a) == 2 and len(ptrs_b) == 1
    for x, y in zip(out_a, out_b):
        for u, v in zip(x, y):
            assert torch.equal(u, v)
    # graph capture needs CUDA; on the host neither mode claims it
    assert not env_a.graph_capturable and not env_b.graph_capturable
