"""Semantics of the PyTorch path checked against hand computation or the upstream reference, on the themes of
upstream's own unit tests: time-out bootstrap, the adaptive learning-rate rule, minibatch coverage and partition
checks, distribution formulas, RND weight schedules and checkpoint resume, legacy checkpoints, RNN reset / detach /
sequential consistency, runner determinism, bucketed gradient reduction and distillation replicas over gloo."""

import copy
import math
import os
import socket

import pytest
import torch

from helpers import ppo_cfg, small_env
from tt_rsl_rl_b200.storage import RolloutStorage
from tt_rsl_rl_b200.utils.tensordict import TensorDict


def _runner(cfg=None, env=None, seed=0):
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    torch.manual_seed(seed)
    return OnPolicyRunner(env or small_env(16), copy.deepcopy(cfg or ppo_cfg()), log_dir=None, device="cpu")


# ---- PPO step semantics -------------------------------------------------------------------------------------------------
def test_timeout_bootstrap_adds_the_discounted_value():
    runner = _runner()
    alg, env = runner.alg, runner.env
    obs = env.get_observations()
    alg.act(obs)
    values = alg.transition.values.clone()
    rewards = torch.arange(16, dtype=torch.float32)
    time_outs = (torch.arange(16) % 3 == 0).float()
    alg.process_env_step(obs, rewards, torch.zeros(16), {"time_outs": time_outs})
    want = rewards + alg.gamma * values[:, 0] * time_outs
    torch.testing.assert_close(alg.storage.rewards[0, :, 0], want)


class _KLStub:
    old_distribution_params = None


@pytest.mark.parametrize("kl,lr0,expect", [
    (0.05, 1e-3, 1e-3 / 1.5),  # above 2 x desired: divide
    (0.05, 1.2e-5, 1e-5),  # ... with a floor
    (0.001, 1e-3, 1.5e-3),  # below desired / 2: multiply
    (0.001, 9e-3, 1e-2),  # ... with a ceiling
    (0.01, 1e-3, 1e-3),  # inside the band: unchanged
    (0.0, 1e-3, 1e-3),  # exactly zero (first minibatch): unchanged
])
def test_adaptive_learning_rate_branches(kl, lr0, expect):
    runner = _runner(ppo_cfg(schedule="adaptive", desired_kl=0.01))
    alg = runner.alg
    alg.learning_rate = lr0
    alg.actor.get_kl_divergence = lambda old, new: torch.full((4,), kl)
    alg._adapt_learning_rate(_KLStub(), ())
    assert alg.learning_rate == pytest.approx(expect)
    assert all(g["lr"] == pytest.approx(expect) for g in alg.optimizer.param_groups)


# ---- storage ------------------------------------------------------------------------------------------------------------
def _filled_storage(N=6, T=4, dones=None):
    obs = TensorDict({"policy": torch.zeros(N, 2)}, batch_size=[N])
    st = RolloutStorage("rl", N, T, obs, [1], "cpu")
    for t in range(T):
        tr = RolloutStorage.Transition()
        ids = (t * N + torch.arange(N)).float()
        tr.observations = TensorDict({"policy": ids[:, None].repeat(1, 2)}, batch_size=[N])
        tr.actions = ids[:, None]
        tr.rewards = torch.zeros(N)
        tr.dones = torch.zeros(N) if dones is None else dones[t]
        tr.values = ids[:, None]
        tr.actions_log_prob = torch.zeros(N)
        tr.distribution_params = (ids[:, None], torch.ones(N, 1))
        st.add_transition(tr)
    return st


def test_minibatches_visit_every_sample_once_per_epoch():
    st = _filled_storage()
    seen = []
    for b in st.mini_batch_generator(num_mini_batches=4, num_epochs=3):
        seen.append(b.observations["policy"][:, 0])
        assert torch.equal(b.observations["policy"][:, 0], b.actions[:, 0])  # fields stay aligned
    assert len(seen) == 12
    for e in range(3):
        epoch = torch.cat(seen[4 * e: 4 * e + 4]).sort().values
        assert torch.equal(epoch, torch.arange(24.0))
    with pytest.raises(OverflowError):
        st.add_transition(RolloutStorage.Transition())


@pytest.mark.parametrize("bad", [0, 25])
def test_invalid_partitions_are_rejected(bad):
    st = _filled_storage()
    with pytest.raises(ValueError):
        next(st.mini_batch_generator(num_mini_batches=bad, num_epochs=1))
    if bad > 6:
        with pytest.raises(ValueError):
            next(st.recurrent_mini_batch_generator(num_mini_batches=bad, num_epochs=1))


def test_recurrent_minibatches_cover_every_environment_once():
    N, T = 6, 4
    dones = [torch.tensor([0, 1, 0, 0, 1, 0.0]), torch.zeros(N), torch.tensor([1, 0, 0, 1, 0, 0.0]), torch.zeros(N)]
    st = _filled_storage(N, T, dones)
    envs = []
    for b in st.recurrent_mini_batch_generator(num_mini_batches=3, num_epochs=1):
        assert b.actions.shape[:2] == (T, 2)
        envs.append(b.actions[0, :, 0].long())
        # every trajectory column starts at a rollout start or right after a done
        assert bool(b.masks[0].all())
    assert torch.equal(torch.cat(envs).sort().values, torch.arange(N))


# ---- distributions --------------------------------------------------------------------------------------------------------
def test_gaussian_formulas_and_std_clamp():
    from tt_rsl_rl_b200.modules.distribution import GaussianDistribution

    d = GaussianDistribution(3, init_std=0.5, std_range=(0.1, 0.4))
    mu = torch.tensor([[0.0, 1.0, -1.0]])
    d.update(mu)
    std = torch.full((1, 3), 0.4)  # the init value 0.5 is clamped into [0.1, 0.4]
    torch.testing.assert_close(d.std, std)
    x = torch.tensor([[0.1, 0.5, -1.2]])
    want = (-(x - mu) ** 2 / (2 * std ** 2) - torch.log(std) - 0.5 * math.log(2 * math.pi)).sum(-1)
    torch.testing.assert_close(d.log_prob(x), want)
    torch.testing.assert_close(d.entropy, (0.5 + 0.5 * math.log(2 * math.pi) + torch.log(std)).sum(-1))
    old = (mu + 0.1, std * 1.5)
    kl = (torch.log(std / old[1]) + (old[1] ** 2 + (old[0] - mu) ** 2) / (2 * std ** 2) - 0.5).sum(-1)
    torch.testing.assert_close(d.kl_divergence(old, (mu, std)), kl)


def test_beta_distribution_matches_torch(ref):
    from rsl_rl.modules.distribution import BetaDistribution as RefBeta

    from tt_rsl_rl_b200.modules.distribution import BetaDistribution

    torch.manual_seed(0)
    ours, theirs = BetaDistribution(4), RefBeta(4)
    out = torch.randn(5, *([ours.input_dim] if isinstance(ours.input_dim, int) else ours.input_dim))
    ours.update(out)
    theirs.update(out)
    x = torch.rand(5, 4) * 1.8 - 0.9
    torch.testing.assert_close(ours.log_prob(x), theirs.log_prob(x))
    torch.testing.assert_close(ours.entropy, theirs.entropy)
    torch.testing.assert_close(ours.mean, theirs.mean)


# ---- RND ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("schedule", [
    {"mode": "constant"},
    {"mode": "step", "final_step": 5, "final_value": 0.1},
    {"mode": "linear", "initial_step": 2, "final_step": 8, "final_value": 0.0},
])
def test_rnd_weight_schedules_match_reference(ref, schedule):
    from rsl_rl.extensions import RandomNetworkDistillation as RefRND

    from tt_rsl_rl_b200.extensions import RandomNetworkDistillation

    kw = dict(num_states=3, obs_groups={"rnd_state": ["policy"]}, num_outputs=2, predictor_hidden_dims=[4],
              target_hidden_dims=[4], weight=1.0, weight_schedule=dict(schedule))
    ours, theirs = RandomNetworkDistillation(**kw), RefRND(**kw)
    obs = TensorDict({"policy": torch.randn(2, 3)}, batch_size=[2])
    import tensordict as ref_td

    ref_obs = ref_td.TensorDict({"policy": obs["policy"]}, batch_size=[2])
    for _ in range(10):
        ours.get_intrinsic_reward(obs)
        theirs.get_intrinsic_reward(ref_obs)
        assert ours.weight == pytest.approx(theirs.weight)


def test_rnd_counter_survives_save_and_load(tmp_path):
    cfg = ppo_cfg()
    cfg["algorithm"]["rnd_cfg"] = {"weight": 1.0, "num_outputs": 4, "predictor_hidden_dims": [8],
                                   "target_hidden_dims": [8], "weight_schedule": {"mode": "step", "final_step": 30,
                                                                                  "final_value": 0.2}}
    r1 = _runner(cfg)
    r1.learn(2)
    counter = r1.alg.rnd.update_counter
    assert counter == 2 * cfg["num_steps_per_env"]
    r1.save(str(tmp_path / "m.pt"))
    d = torch.load(tmp_path / "m.pt", weights_only=False)
    assert d["rnd_update_counter"] == counter and "rnd_state_dict" in d and "rnd_optimizer_state_dict" in d
    r2 = _runner(cfg, seed=1)
    r2.load(str(tmp_path / "m.pt"))
    assert r2.alg.rnd.update_counter == counter
    for a, b in zip(r1.alg.rnd.predictor.parameters(), r2.alg.rnd.predictor.parameters()):
        torch.testing.assert_close(a, b)
    # checkpoints written without the counter (older upstream) load with the counter at zero
    del d["rnd_update_counter"]
    torch.save(d, tmp_path / "old.pt")
    r3 = _runner(cfg, seed=2)
    r3.load(str(tmp_path / "old.pt"))
    assert r3.alg.rnd.update_counter == 0


def test_legacy_model_state_dict_checkpoint_loads(tmp_path):
    r1 = _runner()
    d = r1.alg.save()
    legacy = {"model_state_dict": {}, "optimizer_state_dict": d["optimizer_state_dict"], "iter": 7, "infos": None}
    for k, v in d["actor_state_dict"].items():
        if k.startswith("mlp."):
            legacy["model_state_dict"]["actor." + k[4:]] = v
        elif k.startswith("obs_normalizer."):
            legacy["model_state_dict"]["actor_obs_normalizer." + k.split(".", 1)[1]] = v
        elif k == "distribution.std_param":
            legacy["model_state_dict"]["std"] = v
    for k, v in d["critic_state_dict"].items():
        if k.startswith("mlp."):
            legacy["model_state_dict"]["critic." + k[4:]] = v
        elif k.startswith("obs_normalizer."):
            legacy["model_state_dict"]["critic_obs_normalizer." + k.split(".", 1)[1]] = v
    torch.save(legacy, tmp_path / "legacy.pt")
    r2 = _runner(seed=5)
    r2.load(str(tmp_path / "legacy.pt"))
    assert r2.current_learning_iteration == 7
    obs = r1.env.get_observations()
    torch.testing.assert_close(r2.get_inference_policy()(obs), r1.get_inference_policy()(obs))


# ---- RNN ------------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("rnn_type", ["gru", "lstm"])
def test_rnn_reset_detach_and_sequential_consistency(rnn_type):
    from tt_rsl_rl_b200.modules.rnn import RNN

    torch.manual_seed(0)
    rnn = RNN(3, hidden_dim=5, num_layers=2, type=rnn_type)
    xs = torch.randn(6, 4, 3)
    # step by step (rollout mode) equals the whole sequence through torch's module
    steps = torch.stack([rnn(xs[t]).squeeze(0) for t in range(6)])
    rnn.reset()
    full, _ = rnn.rnn(xs)
    torch.testing.assert_close(steps, full)
    # reset of environment 1 zeroes only its state
    rnn.reset()
    rnn(xs[0])
    h = rnn.hidden_state[0] if rnn.is_lstm else rnn.hidden_state
    assert bool((h[:, 1] != 0).any())
    rnn.reset(torch.tensor([0, 1, 0, 0]))
    h = rnn.hidden_state[0] if rnn.is_lstm else rnn.hidden_state
    assert bool((h[:, 1] == 0).all()) and bool((h[:, 0] != 0).any())
    # detaching cuts the graph without changing values
    out = rnn(xs[1].requires_grad_())
    before = (rnn.hidden_state[0] if rnn.is_lstm else rnn.hidden_state).clone()
    rnn.detach_hidden_state()
    after = rnn.hidden_state[0] if rnn.is_lstm else rnn.hidden_state
    assert not after.requires_grad and torch.equal(before, after) and out.requires_grad


@pytest.mark.parametrize("rnn_type", ["gru", "lstm"])
def test_rnn_model_jit_export_keeps_state(rnn_type, tmp_path):
    from tt_rsl_rl_b200.models import RNNModel

    torch.manual_seed(0)
    obs = TensorDict({"policy": torch.randn(1, 4)}, batch_size=[1])
    m = RNNModel(obs, {"actor": ["policy"]}, "actor", 2, hidden_dims=[8], rnn_type=rnn_type, rnn_hidden_dim=6,
                 distribution_cfg={"class_name": "GaussianDistribution"})
    m.eval()
    jit = torch.jit.script(m.as_jit())
    path = tmp_path / "p.pt"
    jit.save(str(path))
    loaded = torch.jit.load(str(path))
    for _ in range(3):
        x = torch.randn(1, 4)
        with torch.no_grad():
            want = m(TensorDict({"policy": x}, batch_size=[1]))
        torch.testing.assert_close(loaded(x), want)
    loaded.reset()
    m.reset()
    x = torch.randn(1, 4)
    with torch.no_grad():
        torch.testing.assert_close(loaded(x), m(TensorDict({"policy": x}, batch_size=[1])))


# ---- runner -----------------------------------------------------------------------------------------------------------------
def test_runner_is_deterministic_for_a_seed():
    def run():
        r = _runner(env=small_env(16, seed=3), seed=11)
        r.learn(3)
        return [p.detach().clone() for p in r.alg.actor.parameters()]

    for a, b in zip(run(), run()):
        assert torch.equal(a, b)


def test_cnn_runner_learns_saves_and_loads(tmp_path):
    from tt_rsl_rl_b200.env.vec_env import VecEnv
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    class ImageEnv(VecEnv):
        num_envs, num_actions, max_episode_length = 8, 2, 10

        def __init__(self):
            self.device = "cpu"
            self.cfg = {}
            self.episode_length_buf = torch.zeros(8, dtype=torch.long)

        def get_observations(self):
            return TensorDict({"policy": torch.randn(8, 3), "camera": torch.rand(8, 1, 8, 8)}, batch_size=[8])

        def step(self, actions):
            self.episode_length_buf += 1
            return self.get_observations(), -actions.square().sum(1), torch.zeros(8), {"time_outs": torch.zeros(8)}

    cnn = {"output_channels": [4], "kernel_size": 3, "stride": 1, "flatten": True}
    cfg = ppo_cfg(hidden=(16,), T=4, epochs=1, mbs=2, critic_group="policy")
    for k in ("actor", "critic"):
        cfg[k].update({"class_name": "CNNModel", "cnn_cfg": cnn})
    cfg["obs_groups"] = {"actor": ["policy", "camera"], "critic": ["policy", "camera"]}
    r = OnPolicyRunner(ImageEnv(), cfg, log_dir=None, device="cpu")
    r.learn(2)
    r.save(str(tmp_path / "c.pt"))
    r2 = OnPolicyRunner(ImageEnv(), copy.deepcopy(cfg), log_dir=None, device="cpu")
    r2.load(str(tmp_path / "c.pt"))
    obs = ImageEnv().get_observations()
    torch.testing.assert_close(r2.get_inference_policy()(obs), r.get_inference_policy()(obs))


# ---- data parallel over gloo --------------------------------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bucket_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from tt_rsl_rl_b200.utils.utils import reduce_gradients_in_buckets

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    torch.manual_seed(100 + rank)
    shapes = [(3,), (40,), (7, 5), (2,), (100,)]
    a = [torch.nn.Parameter(torch.zeros(s)) for s in shapes]
    b = [torch.nn.Parameter(torch.zeros(s)) for s in shapes]
    for i, (p, q) in enumerate(zip(a, b)):
        if i == 3:
            continue  # a parameter without a gradient
        p.grad = torch.randn(p.shape)
        q.grad = p.grad.clone()
    reduce_gradients_in_buckets(a, world, bucket_mb=256 / 2**20)  # 256-byte buckets: packing and slicing
    reduce_gradients_in_buckets(b, world, bucket_mb=64.0)  # everything in one bucket
    torch.save({"a": [p.grad for p in a], "b": [q.grad for q in b]}, os.path.join(out_dir, f"{rank}.pt"))
    dist.destroy_process_group()


def test_tiny_buckets_equal_one_bucket_and_the_mean(tmp_path):
    torch.multiprocessing.spawn(_bucket_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (torch.load(tmp_path / f"{r}.pt") for r in range(2))
    for ga, gb, ga1 in zip(r0["a"], r0["b"], r1["a"]):
        if ga is None:
            assert gb is None and ga1 is None
            continue
        torch.testing.assert_close(ga, gb)
        torch.testing.assert_close(ga, ga1)
    torch.manual_seed(100)
    g0 = [torch.randn(s) for s in [(3,), (40,), (7, 5)]]
    torch.manual_seed(101)
    g1 = [torch.randn(s) for s in [(3,), (40,), (7, 5)]]
    for k in range(3):
        torch.testing.assert_close(r0["a"][k], (g0[k] + g1[k]) / 2)


def _distill_worker(rank, world, port, out_dir, reduce):
    import torch.distributed as dist

    from tt_rsl_rl_b200.runners import DistillationRunner

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    cfg = {
        "num_steps_per_env": 4, "save_interval": 1000,
        "obs_groups": {"student": ["policy"], "teacher": ["policy", "critic"]},
        "student": {"class_name": "MLPModel", "hidden_dims": [16], "obs_normalization": True,
                    "distribution_cfg": {"class_name": "GaussianDistribution"}},
        "teacher": {"class_name": "MLPModel", "hidden_dims": [16]},
        "algorithm": {"class_name": "Distillation", "num_learning_epochs": 1, "gradient_length": 2,
                      "learning_rate": 1e-2},
    }
    torch.manual_seed(0)
    runner = DistillationRunner(small_env(8, seed=rank), cfg, log_dir=None, device="cpu")
    runner.alg.teacher_loaded = True
    if not reduce:
        runner.alg.reduce_parameters = lambda: None
    runner.learn(2)
    torch.save([p.detach() for p in runner.alg.student.parameters()], os.path.join(out_dir, f"{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("reduce", [True, False])
def test_distillation_replicas_stay_identical_only_with_reduction(tmp_path, reduce):
    torch.multiprocessing.spawn(_distill_worker, args=(2, _free_port(), str(tmp_path), reduce), nprocs=2, join=True)
    p0, p1 = (torch.load(tmp_path / f"{r}.pt") for r in range(2))
    same = all(torch.equal(a, b) for a, b in zip(p0, p1))
    assert same == reduce


def test_reduce_parameters_on_one_rank_is_the_identity():
    """With one rank the bucketed mean leaves every gradient as it was (the all-reduce of one rank is stubbed, as
    no process group exists here)."""
    runner = _runner()
    alg = runner.alg
    for p in alg.actor.parameters():
        p.grad = torch.full_like(p, 0.5)
    alg.gpu_world_size = 1
    calls = []
    orig = torch.distributed.all_reduce
    torch.distributed.all_reduce = lambda t, op=None: calls.append(t.numel())
    try:
        alg.reduce_parameters()
    finally:
        torch.distributed.all_reduce = orig
    assert sum(calls) == sum(p.numel() for p in alg.actor.parameters()) + sum(
        p.numel() for p in alg.critic.parameters() if p.grad is not None)
    assert all(bool((p.grad == 0.5).all()) for p in alg.actor.parameters())


# ---- loss tables, mixed precision, shared encoders ------------------------------------------------------------------------
def _direct_ppo(**kw):
    from tt_rsl_rl_b200.algorithms import PPO
    from tt_rsl_rl_b200.models import MLPModel

    torch.manual_seed(0)
    N, T, A = 8, 4, 3
    obs = TensorDict({"policy": torch.randn(N, 5)}, batch_size=[N])
    groups = {"actor": ["policy"], "critic": ["policy"]}
    actor = MLPModel(obs, groups, "actor", A, hidden_dims=[16],
                     distribution_cfg={"class_name": "GaussianDistribution", "init_std": 1.0})
    critic = MLPModel(obs, groups, "critic", 1, hidden_dims=[16])
    ppo = PPO(actor, critic, RolloutStorage("rl", N, T, obs, [A]), **kw)
    ppo.train_mode()
    for _ in range(T):
        ppo.act(obs)
        ppo.process_env_step(obs, torch.randn(N), torch.zeros(N), {})
    ppo.compute_returns(obs)
    return ppo


@pytest.mark.parametrize("advantage,ratio,expected", [(1.0, 1.5, -1.2), (-1.0, 0.5, 0.8), (1.0, 0.5, -0.5)])
def test_surrogate_clipping_table(advantage, ratio, expected):
    """-min(A r, A clip(r, 0.8, 1.2)) for ratios outside the clip range, positive and negative advantages."""
    ppo = _direct_ppo(num_learning_epochs=1, num_mini_batches=1, schedule="fixed")
    ppo.storage.actions_log_prob.sub_(math.log(ratio))
    ppo.storage.advantages.fill_(advantage)
    assert ppo.update()["surrogate"] == pytest.approx(expected, rel=1e-5)


@pytest.mark.parametrize("clipped,offset,expected", [(True, 0.0, 0.64), (False, 0.0, 0.0), (True, -1.0, 1.0)])
def test_value_clipping_table(clipped, offset, expected):
    """Old values 1 below the prediction: the clipped estimate moves only 0.2 towards it."""
    ppo = _direct_ppo(num_learning_epochs=1, num_mini_batches=1, schedule="fixed", use_clipped_value_loss=clipped)
    ppo.storage.returns.copy_(ppo.storage.values + offset)
    ppo.storage.values.sub_(1.0)
    assert ppo.update()["value"] == pytest.approx(expected, abs=1e-5)


def test_mixed_precision_is_opt_in_and_updates():
    assert _direct_ppo().use_mixed_precision is False
    ppo = _direct_ppo(use_mixed_precision=True, schedule="fixed")
    before = [p.clone() for p in ppo.actor.parameters()]
    losses = ppo.update()
    assert all(math.isfinite(v) for v in losses.values())
    assert any(not torch.equal(b, a) for b, a in zip(before, ppo.actor.parameters()))


def test_shared_cnn_encoder_is_stepped_once():
    from tt_rsl_rl_b200.algorithms import PPO
    from tt_rsl_rl_b200.models import CNNModel

    obs = TensorDict({"policy": torch.randn(4, 3), "image": torch.randn(4, 1, 8, 8)}, batch_size=[4])
    groups = {"actor": ["policy", "image"], "critic": ["policy", "image"]}
    cnn_cfg = {"image": {"output_channels": [4], "kernel_size": 3, "stride": 1, "activation": "elu"}}
    actor = CNNModel(obs, groups, "actor", 2, hidden_dims=[8], cnn_cfg=cnn_cfg,
                     distribution_cfg={"class_name": "GaussianDistribution", "init_std": 1.0})
    critic = CNNModel(obs, groups, "critic", 1, hidden_dims=[8], cnns=actor.cnns)
    ppo = PPO(actor, critic, RolloutStorage("rl", 4, 2, obs, [2]), learning_rate=1e-3)
    params = ppo.optimizer.param_groups[0]["params"]
    assert len(params) == len({id(p) for p in params})
    shared = next(actor.cnns.parameters())
    assert any(shared is p for p in critic.parameters())
    before = shared.detach().clone()
    for p in params:
        p.grad = torch.ones_like(p)
    ppo.optimizer.step()
    assert int(ppo.optimizer.state[shared]["step"]) == 1
    assert (before - shared.detach()).abs().max().item() == pytest.approx(1e-3, abs=1e-6)  # one Adam step of lr


# ---- writer lifecycle ----------------------------------------------------------------------------------------------------
def test_writer_lifecycle_on_success_and_on_failure(tmp_path):
    from helpers import RecordingWriter

    cfg = ppo_cfg(T=4)
    cfg["logger"] = {"class_name": "helpers:RecordingWriter"}
    cfg["save_interval"] = 2
    RecordingWriter.events.clear()
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    runner = OnPolicyRunner(small_env(8), copy.deepcopy(cfg), log_dir=str(tmp_path / "a"), device="cpu")
    runner.learn(3)
    kinds = [e[0] for e in RecordingWriter.events]
    assert kinds[0] == "init" and kinds.count("config") == 1 and kinds[-1] == "stop" and "abort" not in kinds
    assert [e[1] for e in RecordingWriter.events if e[0] == "model"] == [0, 2, 2]  # interval saves + the final one
    assert {e[2] for e in RecordingWriter.events if e[0] == "scalar"} == {0, 1, 2}

    class Failing(type(small_env(8))):
        calls = 0

        def step(self, actions):
            Failing.calls += 1
            if Failing.calls > 5:
                raise RuntimeError("simulator crashed")
            return super().step(actions)

    RecordingWriter.events.clear()
    env = small_env(8)
    env.__class__ = Failing
    runner = OnPolicyRunner(env, copy.deepcopy(cfg), log_dir=str(tmp_path / "b"), device="cpu")
    with pytest.raises(RuntimeError, match="simulator crashed"):
        runner.learn(3)
    kinds = [e[0] for e in RecordingWriter.events]
    assert kinds[-1] == "abort" and "stop" not in kinds


# ---- W&B / Neptune writers with fake client modules ------------------------------------------------------------------------
def _fake_wandb(calls):
    import types

    m = types.ModuleType("wandb")
    m.init = lambda **kw: calls.append(("init", kw))
    m.log = lambda data, step=None: calls.append(("log", data, step))
    m.save = lambda path, base_path=None: calls.append(("save", path))
    m.finish = lambda exit_code=0: calls.append(("finish", exit_code))
    m.Video = lambda path, format=None: ("video-object", path)
    m.config = types.SimpleNamespace(update=lambda d: calls.append(("config", d)))
    return m


class _FakeNeptuneRun:
    def __init__(self, calls):
        self.calls = calls

    def __getitem__(self, key):
        calls, outer = self.calls, self

        class Field:
            def log(self, value, step=None):
                calls.append(("log", key, value, step))

            def upload(self, path):
                calls.append(("upload", key, path))

        return Field()

    def __setitem__(self, key, value):
        self.calls.append(("set", key, value))

    def stop(self):
        self.calls.append(("stop",))


def test_wandb_and_neptune_writers_with_fake_clients(tmp_path, monkeypatch):
    import dataclasses
    import sys
    import types

    from tt_rsl_rl_b200.utils import NeptuneLogWriter, WandbLogWriter

    @dataclasses.dataclass
    class EnvCfg:
        dt: float = 0.02

    calls = []
    monkeypatch.setitem(sys.modules, "wandb", _fake_wandb(calls))
    monkeypatch.setenv("WANDB_USERNAME", "someone")
    w = WandbLogWriter(str(tmp_path / "wb" / "run_7"), project_name="proj")
    w.add_scalar("Loss/value", 1.5, 3)
    w.store_config(EnvCfg(), {"num_steps_per_env": 24})
    w.save_video(tmp_path / "v.mp4", 4)
    w.stop()
    init = calls[0][1]
    assert init["project"] == "proj" and init["entity"] == "someone" and init["name"] == "run_7"
    assert ("log", {"Loss/value": 1.5}, 3) in calls
    assert ("config", {"train_cfg": {"num_steps_per_env": 24}}) in calls and ("config", {"env_cfg": {"dt": 0.02}}) in calls
    assert any(c[0] == "log" and "video" in c[1] for c in calls) and calls[-1] == ("finish", 0)
    assert any(p.name.startswith("events.out.tfevents") for p in (tmp_path / "wb" / "run_7").iterdir())  # TensorBoard copy

    calls.clear()
    neptune = types.ModuleType("neptune")
    neptune.init_run = lambda project, api_token, **kw: (calls.append(("init", project, api_token)), _FakeNeptuneRun(calls))[1]
    monkeypatch.setitem(sys.modules, "neptune", neptune)
    monkeypatch.delenv("NEPTUNE_API_TOKEN", raising=False)
    with pytest.raises(KeyError, match="NEPTUNE_API_TOKEN"):
        NeptuneLogWriter(str(tmp_path / "nep" / "run_8"), project_name="proj")
    monkeypatch.setenv("NEPTUNE_API_TOKEN", "tok")
    monkeypatch.setenv("NEPTUNE_USERNAME", "me")
    n = NeptuneLogWriter(str(tmp_path / "nep" / "run_8"), project_name="proj")
    n.add_scalar("Train/mean_reward/time", 2.0, 5)
    n.store_config({"a": 1}, {"b": 2})
    n.save_model(str(tmp_path / "model_5.pt"), 5)
    n.save_file(str(tmp_path / "repo.diff"))
    n.stop()
    assert ("init", "me/proj", "tok") in calls and ("log", "log_dir", "run_8", None) in calls
    assert ("log", "Train/mean_reward_time", 2.0, 5) in calls
    assert ("set", "train_cfg", {"b": 2}) in calls and ("set", "env_cfg", {"a": 1}) in calls
    assert ("upload", "model/saved_model_5", str(tmp_path / "model_5.pt")) in calls
    assert ("upload", "git_diff/repo", str(tmp_path / "repo.diff")) in calls and calls[-1] == ("stop",)


def test_play_evaluates_the_newest_checkpoint(tmp_path):
    from tt_rsl_rl_b200.runners import play
    from tt_rsl_rl_b200.testing import reference as R

    import dataclasses

    spec = dataclasses.replace(R.SPECS["cartpole"], num_envs=64, num_steps=8)
    R.train("cartpole", 0, str(tmp_path), iterations=2, spec=spec)
    runner, _, _ = R.build_runner("cartpole", 0, None, spec)  # a checkpoint the CSV run did not write
    runner.save(str(tmp_path / "model_7.pt"))
    import contextlib
    import io
    import json

    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        assert play.main(["--run-dir", str(tmp_path), "--env", "cartpole", "--num-envs", "32", "--steps", "300",
                          "--device", "cpu", "--export-jit", str(tmp_path / "exported")]) == 0
    out = json.loads(buf.getvalue().strip().splitlines()[-1])
    assert out["checkpoint"].endswith("model_7.pt") and out["episodes"] > 0 and out["mean_length"] > 0
    assert (tmp_path / "exported" / "policy.pt").exists()


def test_checkpoint_loads_after_a_rollout_with_rnd_reward_normalisation(tmp_path):
    """The RND reward normaliser is updated inside the rollout (inference mode); its buffers stay ordinary tensors, so
    loading a checkpoint into a runner that has already trained works."""
    cfg = ppo_cfg(T=4)
    cfg["algorithm"]["rnd_cfg"] = {"weight": 1.0, "num_outputs": 4, "predictor_hidden_dims": [8],
                                   "target_hidden_dims": [8], "reward_normalization": True,
                                   "state_normalization": True}
    r = _runner(cfg)
    r.learn(2)
    assert not r.alg.rnd.reward_normalizer.emp_norm._std.is_inference()
    r.save(str(tmp_path / "m.pt"))
    r.learn(1)
    r.load(str(tmp_path / "m.pt"))
    assert r.current_learning_iteration == 1


def test_torch_path_stores_the_observations_it_acted_on_with_an_in_place_environment():
    """An environment that rewrites its observation tensors in place (as graph-capturable ones do) still gives the
    PyTorch path's storage the observations each action was computed from."""
    from tt_rsl_rl_b200.env.vec_env import VecEnv

    class InPlaceEnv(VecEnv):
        graph_capturable = True
        num_envs, num_actions, max_episode_length = 4, 2, 100

        def __init__(self):
            self.device = "cpu"
            self.cfg = {}
            self.episode_length_buf = torch.zeros(4, dtype=torch.long)
            self.t = 0
            self.buf = torch.zeros(4, 3)
            self.obs = TensorDict({"policy": self.buf, "critic": self.buf}, batch_size=[4])
            self.seen = []

        def get_observations(self):
            return self.obs

        def step(self, actions):
            self.t += 1
            self.buf.fill_(float(self.t))  # in place
            return self.obs, torch.zeros(4), torch.zeros(4), {"time_outs": torch.zeros(4)}

    env = InPlaceEnv()
    r = _runner(ppo_cfg(T=4), env=env)
    r.alg.update = lambda: {}  # keep the stored rollout
    r.alg.storage.clear = lambda: None
    r.learn(1)
    stored = r.alg.storage.observations["policy"][:, 0, 0]
    assert stored.tolist() == [0.0, 1.0, 2.0, 3.0]  # step t stores the observation of step t, not t + 1
