"""Data-parallel correctness of the fused CUDA engine on 2+ GPUs (one process per GPU).

* **N GPUs vs 1 GPU on the union minibatch.** Identical synthetic rollouts are injected: the union rollout has
  ``T x N_u`` samples, rank ``r`` of ``W`` holds environments ``[r N_u / W, (r + 1) N_u / W)`` of every step, and the
  sample order is the identity, so minibatch ``k`` of rank ``r`` is the ``r``-th slice of union minibatch ``k``. The
  data-parallel step (local loss and gradient, rank-averaged gradient, KL mean, per-model clip, Adam) then equals one
  GPU stepping on the union minibatch up to the floating-point summation order. Advantages are injected already
  normalised (the rank-local normalisation of ``compute_returns`` is tested elsewhere); the observation normaliser
  update after the epochs is global over ranks on both sides. The comparison is in function space: the deviation
  of the policy means and values of the ``W``-GPU run from the 1-GPU run, relative to how far the update moved them.
  Counterpart of the reference's ``rsl_rl_tt/testing/mc_equiv.py:64-125`` and ``tests/tt/test_tt_multichip.py:95``.
* **A corrupted replica is detected.** With ``replica_check_interval = 1`` one rank's parameter is changed on the
  host between two iterations; the next check raises ``ReplicaDivergenceError`` on every rank
  (``tests/tt/test_tt_multichip.py:161`` in the reference).

Skipped when fewer than two GPUs are visible. NVLS is switched off for NCCL (bootstrap only).
"""

import json
import os
import socket
import tempfile
import types

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

T, N_UNION, A, D_A, D_C = 2, 2048, 12, 48, 51
# Function-space bound of the W-GPU vs 1-GPU deviation. Sources of difference: the order of the fp32 sums of the
# weight gradients (split-K partials over different row counts, then the rank sum) and of the normaliser moments,
# ~1e-6 of the update size, and bf16 weight shadows that round the other way after a parameter moved by that much
# (a few weights in the network by one bf16 unit). Measured on B200 at 2 ranks: 3.1e-7 (policy) and 1.1e-6 (value);
# the bound is about three times that with room for more ranks (longer rank sums).
TOL = 1e-5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _models(hetero: bool):
    from tt_rsl_rl_b200.models import MLPModel
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    obs = TensorDict({"policy": torch.zeros(4, D_A), "critic": torch.zeros(4, D_C)}, batch_size=[4])
    groups = {"actor": ["policy"], "critic": ["critic"]}
    dist = {"class_name": "HeteroscedasticGaussianDistribution" if hetero else "GaussianDistribution",
            "init_std": 1.0}
    torch.manual_seed(0)  # identical initial weights in every process
    actor = MLPModel(obs, groups, "actor", A, hidden_dims=[256, 128, 64], obs_normalization=True,
                     distribution_cfg=dist)
    critic = MLPModel(obs, groups, "critic", 1, hidden_dims=[256, 128, 64], obs_normalization=True)
    return actor, critic


def _union_rollout(actor, critic, hetero: bool):
    """The union rollout ``[T, N_u, .]`` on the host, built from the initial models so that ratios and the KL are
    non-trivial (the stored policy is a slightly moved copy of the current one)."""
    g = torch.Generator().manual_seed(1234)
    obs_a = torch.randn(T, N_UNION, D_A, generator=g) * 1.5 + 0.3
    obs_c = torch.cat([obs_a, torch.randn(T, N_UNION, D_C - D_A, generator=g)], dim=-1)
    with torch.no_grad():
        td = _td(obs_a.flatten(0, 1), obs_c.flatten(0, 1))
        mean = actor(td).reshape(T, N_UNION, A)
        actor(td, stochastic_output=True)  # sets the distribution's std
        std = actor.output_std.detach().expand(T * N_UNION, A).reshape(T, N_UNION, A).clone()
        if hetero:  # the stored per-row std differs from the current one
            std = std * (1 + 0.1 * torch.rand(T, N_UNION, A, generator=g))
        value = critic(td).reshape(T, N_UNION, 1)
    actions = mean + std * torch.randn(T, N_UNION, A, generator=g)
    old_mean = mean + 0.05 * torch.randn(T, N_UNION, A, generator=g)
    old_logp = torch.distributions.Normal(old_mean, std).log_prob(actions).sum(-1, keepdim=True)
    values = value + 0.1 * torch.randn(T, N_UNION, 1, generator=g)
    returns = value + torch.randn(T, N_UNION, 1, generator=g)
    adv = torch.randn(T, N_UNION, 1, generator=g)
    adv = (adv - adv.mean()) / (adv.std() + 1e-8)
    return dict(obs_a=obs_a, obs_c=obs_c, actions=actions, mean=old_mean, std=std, logp=old_logp, values=values,
                returns=returns, adv=adv, rewards=torch.zeros(T, N_UNION, 1), dones=torch.zeros(T, N_UNION, 1))


def _td(obs_a, obs_c):
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    return TensorDict({"policy": obs_a, "critic": obs_c}, batch_size=[obs_a.shape[0]])


def _storage_slice(u: dict, lo: int, hi: int, device):
    """A storage-like view of environments ``[lo, hi)`` of the union rollout (the fields ``load_rollout`` reads)."""
    d = {k: v[:, lo:hi].to(device) for k, v in u.items()}
    obs = types.SimpleNamespace(flatten=lambda a, b: {"policy": d["obs_a"].flatten(0, 1),
                                                      "critic": d["obs_c"].flatten(0, 1)})
    return types.SimpleNamespace(observations=obs, distribution_params=(d["mean"], d["std"]), actions=d["actions"],
                                 actions_log_prob=d["logp"], values=d["values"], rewards=d["rewards"],
                                 dones=d["dones"], returns=d["returns"], advantages=d["adv"])


def run_union_step(rank: int, world: int, hetero: bool) -> dict:
    """One update (2 epochs x 2 minibatches) of the fused engine on this rank's share of the union rollout."""
    from tt_rsl_rl_b200.algorithms import PPO

    device = f"cuda:{rank}"
    actor, critic = _models(hetero)
    u = _union_rollout(actor, critic, hetero)
    g = torch.Generator().manual_seed(99)
    probe_a = torch.randn(4096, D_A, generator=g)
    probe = _td(probe_a, torch.cat([probe_a, torch.randn(4096, D_C - D_A, generator=g)], -1)).to(device)
    n_local = N_UNION // world
    multi = {"global_rank": rank, "local_rank": rank, "world_size": world} if world > 1 else None
    alg = PPO(actor, critic, None, num_learning_epochs=2, num_mini_batches=T, learning_rate=1e-3,
              schedule="adaptive", desired_kl=0.01, device=device, multi_gpu_cfg=multi,
              b200_cfg={"engine": "cuda", "graphs": False, "comm_timeout_ms": 20000},
              num_steps_per_env=T, num_envs=n_local)
    eng = alg.engine
    assert eng is not None and (world == 1 or eng.comm is not None)
    if world > 1:
        alg.broadcast_parameters()
    eng.load_rollout(_storage_slice(u, rank * n_local, (rank + 1) * n_local, device))
    eng.perm_override = torch.arange(T * n_local, dtype=torch.int32, device=device)
    with torch.no_grad():
        before = (alg.actor(probe).cpu(), alg.critic(probe).cpu())
    losses = alg.update()
    with torch.no_grad():
        after = (alg.actor(probe).cpu(), alg.critic(probe).cpu())
    return {"mean_before": before[0], "value_before": before[1], "mean_after": after[0], "value_after": after[1],
            "lr": alg.learning_rate, "losses": losses, "norm_mean": alg.actor.obs_normalizer._mean.cpu().clone(),
            "status": eng.status.cpu().tolist()}


def _equiv_worker(rank: int, world: int, port: int, out_dir: str, hetero: bool) -> None:
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                         timeout=datetime.timedelta(seconds=60))
    try:
        res = run_union_step(rank, world, hetero)
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
        torch.distributed.barrier()
    finally:
        torch.distributed.destroy_process_group()


def _deviation(multi: dict, single: dict) -> tuple[float, float]:
    dm = (multi["mean_after"] - single["mean_after"]).norm() / (single["mean_after"] - single["mean_before"]).norm()
    dv = (multi["value_after"] - single["value_after"]).norm() / (single["value_after"]
                                                                  - single["value_before"]).norm()
    return float(dm), float(dv)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("hetero", [False, True])
def test_n_gpus_equal_one_gpu_on_the_union_minibatch(hetero):
    single = run_union_step(0, 1, hetero)
    assert single["status"][0] == 0
    for world in sorted({2, min(torch.cuda.device_count(), 4)}):
        out_dir = tempfile.mkdtemp()
        torch.multiprocessing.spawn(_equiv_worker, args=(world, _free_port(), out_dir, hetero), nprocs=world,
                                    join=True)
        res = [torch.load(os.path.join(out_dir, f"rank{r}.pt")) for r in range(world)]
        for r in res:
            assert r["status"][0] == 0
            # replicas agree bit for bit, so rank 0 stands for all
            assert torch.equal(r["mean_after"], res[0]["mean_after"])
            assert torch.equal(r["value_after"], res[0]["value_after"])
        # the starting point is the same function on both sides
        assert torch.equal(res[0]["mean_before"], single["mean_before"])
        dm, dv = _deviation(res[0], single)
        print(f"\n[n-vs-1] hetero={hetero} world={world}: policy deviation {dm:.3e}, value deviation {dv:.3e} "
              f"(of the update); lr {res[0]['lr']:.6g} vs {single['lr']:.6g}")
        assert dm < TOL and dv < TOL, (world, dm, dv)
        assert res[0]["lr"] == pytest.approx(single["lr"], rel=1e-6)
        torch.testing.assert_close(res[0]["norm_mean"], single["norm_mean"], rtol=1e-5, atol=1e-6)
        for k in ("surrogate", "value", "entropy"):
            assert res[0]["losses"][k] == pytest.approx(single["losses"][k], rel=1e-4, abs=1e-6), k


def test_rank_slices_tile_the_union():
    """Host check of the layout: the ranks' slices of every union minibatch are disjoint and cover it."""
    for world in (1, 2, 4, 8):
        n = N_UNION // world
        rows = sorted(t * N_UNION + r * n + j for r in range(world) for t in range(T) for j in range(n))
        assert rows == list(range(T * N_UNION))


def _replica_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank), "NCCL_NVLS_ENABLE": "0"})
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                         timeout=datetime.timedelta(seconds=60))
    from tt_rsl_rl_b200.env import LinearGaussianVecEnv
    from tt_rsl_rl_b200.parallel import ReplicaDivergenceError
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    class CorruptingEnv(LinearGaussianVecEnv):
        """Calls ``corrupt`` once, from the host, between two environment steps of the second iteration."""

        corrupt = None
        calls = 0

        def step(self, actions):
            self.calls += 1
            if self.calls == T_STEPS + 3 and self.corrupt is not None:
                self.corrupt()
            return super().step(actions)

    T_STEPS = 8
    cfg = {"num_steps_per_env": T_STEPS, "save_interval": 1000,
           "obs_groups": {"actor": ["policy"], "critic": ["critic"]},
           "algorithm": {"class_name": "PPO", "num_learning_epochs": 1, "num_mini_batches": 2,
                         "b200_cfg": {"comm_timeout_ms": 20000, "engine": "cuda", "replica_check_interval": 1}},
           "actor": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True,
                     "distribution_cfg": {"class_name": "GaussianDistribution", "init_std": 1.0}},
           "critic": {"class_name": "MLPModel", "hidden_dims": [64, 64], "obs_normalization": True}}
    res = {"rank": rank, "raised": None}
    try:
        # the PyTorch-op step (not graph-captured), so the host runs between every two steps
        env = CorruptingEnv(512, obs_dim=48, num_actions=12, privileged_dim=3, device=f"cuda:{rank}",
                            seed=10 + rank, fused=False)
        runner = OnPolicyRunner(env, cfg, log_dir=None, device=f"cuda:{rank}")
        assert runner.alg.engine is not None and runner.alg.engine.comm is not None
        if rank == world - 1:  # corrupt this rank's replica during the second iteration's rollout
            weight = runner.alg.actor.mlp[0].weight

            def corrupt():
                with torch.no_grad():
                    weight[0, 0] += 0.5

            env.corrupt = corrupt
        try:
            runner.learn(3)
        except ReplicaDivergenceError as e:
            res["raised"] = str(e)
        torch.cuda.synchronize()
        res["status"] = runner.alg.engine.status.tolist()
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(res, f)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_corrupted_replica_is_detected_on_every_rank():
    world = 2
    out_dir = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_replica_worker, args=(world, _free_port(), out_dir), nprocs=world, join=True)
    res = [json.load(open(os.path.join(out_dir, f"rank{r}.json"))) for r in range(world)]
    for r in res:
        # the first update's check passes, the second one (after the corruption) fails on every rank
        assert r["raised"] is not None and "after update 2" in r["raised"] and "ranks [1]" in r["raised"], r
        assert r["status"][0] == 0
