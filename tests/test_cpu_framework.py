"""Host-only tests of the framework layer: utilities, TensorDict, runner features, data parallelism over gloo and
host-side failure detection. No GPU is used."""

import copy
import os
import socket
import tempfile

import pytest
import torch

from helpers import ppo_cfg, small_env


# ---- utilities ---------------------------------------------------------------------------------------------------------
def test_resolve_callable_forms():
    from tt_rsl_rl_b200.algorithms import PPO
    from tt_rsl_rl_b200.utils import resolve_callable

    assert resolve_callable("PPO") is PPO
    assert resolve_callable("tt_rsl_rl_b200.algorithms:PPO") is PPO
    assert resolve_callable("tt_rsl_rl_b200.algorithms.PPO") is PPO
    assert resolve_callable(PPO) is PPO
    assert resolve_callable("GaussianDistribution").__name__ == "GaussianDistribution"
    with pytest.raises(ValueError):
        resolve_callable("NoSuchThing")
    with pytest.raises(TypeError):
        resolve_callable(3)


def test_resolve_obs_groups_rules():
    from tt_rsl_rl_b200.utils import TensorDict, resolve_obs_groups

    obs = TensorDict({"policy": torch.zeros(2, 3), "critic": torch.zeros(2, 4)}, batch_size=[2])
    g = resolve_obs_groups(obs, {"actor": ["policy"]}, ["actor", "critic"])
    assert g["critic"] == ["critic"]
    g = resolve_obs_groups(obs, {}, ["actor", "rnd_state"])
    assert g == {"actor": ["policy"], "rnd_state": ["policy"]}
    with pytest.raises(ValueError):
        resolve_obs_groups(obs, {"actor": []}, ["actor"])
    with pytest.raises(ValueError):
        resolve_obs_groups(obs, {"actor": ["nope"]}, ["actor"])


def test_activation_and_optimizer_resolution():
    from tt_rsl_rl_b200.utils import resolve_nn_activation, resolve_optimizer

    assert isinstance(resolve_nn_activation("ELU"), torch.nn.ELU)
    assert resolve_optimizer("AdamW") is torch.optim.AdamW
    with pytest.raises(ValueError):
        resolve_nn_activation("bogus")
    with pytest.raises(ValueError):
        resolve_optimizer("bogus")


def test_tensordict_operations():
    from tt_rsl_rl_b200.utils import TensorDict

    td = TensorDict({"a": torch.arange(24.0).view(4, 3, 2), "b": torch.ones(4, 3, 1)}, batch_size=[4, 3])
    assert td.batch_size == torch.Size([4, 3])
    f = td.flatten(0, 1)
    assert f.batch_size == torch.Size([12]) and f["a"].shape == (12, 2)
    sub = f[torch.tensor([0, 5, 7])]
    assert sub.batch_size == torch.Size([3])
    torch.testing.assert_close(sub["a"][1], torch.tensor([10.0, 11.0]))
    td[1].copy_({"a": torch.zeros(3, 2), "b": torch.zeros(3, 1)})
    assert float(td["a"][1].sum()) == 0.0
    cat = torch.cat([f, f])
    assert cat.batch_size == torch.Size([24])
    tr = td.transpose(1, 0)
    assert tr.batch_size == torch.Size([3, 4]) and tr["a"].shape == (3, 4, 2)
    v = tr.reshape(-1, 2)
    assert v.batch_size == torch.Size([6, 2])
    assert td[:, 1:].batch_size == torch.Size([4, 2])
    assert set(td.keys()) == {"a", "b"} and "a" in td
    with pytest.raises(ValueError):
        td["c"] = torch.zeros(5)


def test_feistel_permutation_is_a_bijection():
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    for n in (1, 2, 7, 100, 1000, 4097, 24 * 1001):
        hb = C.feistel_half_bits(n)
        vals = sorted(C.feistel_permute(i, n, hb, 12345) for i in range(n))
        assert vals == list(range(n))
    n = 5000
    hb = C.feistel_half_bits(n)
    a = [C.feistel_permute(i, n, hb, 1) for i in range(50)]
    b = [C.feistel_permute(i, n, hb, 2) for i in range(50)]
    assert a != b  # the key changes the order


# ---- runner features ---------------------------------------------------------------------------------------------------
def test_runner_learn_logs_saves_and_exports(tmp_path):
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    cfg = ppo_cfg()
    cfg["logger"] = {"class_name": "CsvLogWriter"}
    cfg["save_interval"] = 1
    runner = OnPolicyRunner(small_env(), cfg, log_dir=str(tmp_path), device="cpu")
    runner.learn(3)
    assert (tmp_path / "metrics.csv").exists()
    text = (tmp_path / "metrics.csv").read_text().splitlines()
    assert "Loss/surrogate" in text[0] and len(text) >= 3
    assert (tmp_path / "model_2.pt").exists()
    runner.export_policy_to_jit(str(tmp_path), "policy.pt")
    jit = torch.jit.load(str(tmp_path / "policy.pt"))
    x = small_env().get_observations()["policy"]
    with torch.no_grad():
        torch.testing.assert_close(jit(x), runner.get_inference_policy()({"policy": x}))


def test_section_timer_and_runner_sections(tmp_path):
    import time

    from tt_rsl_rl_b200.runners import OnPolicyRunner
    from tt_rsl_rl_b200.utils.timer import SectionTimer

    t = SectionTimer(True, "cpu")
    with t.section("a"):
        time.sleep(0.01)
    with t.section("a"):
        time.sleep(0.01)
    with t.section("b"):
        pass
    out = t.resolve()
    assert set(out) == {"a", "b"} and out["a"] >= 15.0 and t.resolve() == {}
    off = SectionTimer(False, "cpu")
    with off.section("x"):
        pass
    assert off.resolve() == {}
    cfg = ppo_cfg(b200_cfg={"section_timing": True})
    cfg["logger"] = {"class_name": "CsvLogWriter"}
    runner = OnPolicyRunner(small_env(), cfg, log_dir=str(tmp_path), device="cpu")
    runner.learn(2)
    assert set(runner.section_timer.totals) == {"rollout", "returns", "update"}
    csv_text = open(os.path.join(str(tmp_path), "metrics.csv")).read()
    assert "Perf/section_update_ms" in csv_text


def test_runner_tensorboard_default(tmp_path):
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    runner = OnPolicyRunner(small_env(), ppo_cfg(), log_dir=str(tmp_path), device="cpu")
    runner.learn(1)
    assert any(p.name.startswith("events.out.tfevents") for p in tmp_path.iterdir())
    assert (tmp_path / "git").is_dir()


def test_runner_resume_continues_iteration_count(tmp_path):
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    cfg = ppo_cfg()
    r1 = OnPolicyRunner(small_env(), copy.deepcopy(cfg), log_dir=None, device="cpu")
    r1.learn(2)
    r1.save(str(tmp_path / "m.pt"))
    r2 = OnPolicyRunner(small_env(), copy.deepcopy(cfg), log_dir=None, device="cpu")
    r2.load(str(tmp_path / "m.pt"))
    assert r2.current_learning_iteration == 1
    assert r2.alg.learning_rate == pytest.approx(r1.alg.learning_rate)


def test_distillation_runner_requires_teacher(tmp_path):
    from tt_rsl_rl_b200.runners import DistillationRunner, OnPolicyRunner

    cfg = {
        "num_steps_per_env": 8, "save_interval": 100, "obs_groups": {"student": ["policy"], "teacher": ["policy"]},
        "algorithm": {"class_name": "Distillation", "num_learning_epochs": 1, "gradient_length": 4},
        "student": {"class_name": "MLPModel", "hidden_dims": [32, 32],
                    "distribution_cfg": {"class_name": "GaussianDistribution"}},
        "teacher": {"class_name": "MLPModel", "hidden_dims": [32, 32], "obs_normalization": True,
                    "distribution_cfg": {"class_name": "GaussianDistribution"}},
    }
    runner = DistillationRunner(small_env(), copy.deepcopy(cfg), log_dir=None, device="cpu")
    with pytest.raises(ValueError):
        runner.learn(1)
    # an RL checkpoint provides the teacher
    rl_cfg = ppo_cfg(hidden=(32, 32), critic_group="policy")
    rl = OnPolicyRunner(small_env(), rl_cfg, log_dir=None, device="cpu")
    rl.save(str(tmp_path / "rl.pt"))
    runner.load(str(tmp_path / "rl.pt"))
    assert runner.alg.teacher_loaded
    runner.learn(2)


def test_ppo_cpu_with_rnd_symmetry_and_recurrent():
    from tt_rsl_rl_b200.runners import OnPolicyRunner
    from tt_rsl_rl_b200.utils import TensorDict

    def mirror(env, obs=None, actions=None):
        o = a = None
        if obs is not None:
            o = TensorDict({k: torch.cat([v, -v]) for k, v in obs.items()}, batch_size=[2 * obs.batch_size[0]])
        if actions is not None:
            a = torch.cat([actions, -actions])
        return o, a

    cfg = ppo_cfg()
    cfg["algorithm"]["rnd_cfg"] = {"num_outputs": 4, "predictor_hidden_dims": [16], "target_hidden_dims": [16],
                                   "weight": 0.5, "state_normalization": True}
    cfg["algorithm"]["symmetry_cfg"] = {"data_augmentation_func": mirror, "use_data_augmentation": True,
                                        "use_mirror_loss": True, "mirror_loss_coeff": 1.0}
    cfg["obs_groups"]["rnd_state"] = ["critic"]
    runner = OnPolicyRunner(small_env(), cfg, log_dir=None, device="cpu")
    runner.learn(2)
    rcfg = ppo_cfg()
    for m in ("actor", "critic"):
        rcfg[m]["class_name"] = "RNNModel"
        rcfg[m]["rnn_type"] = "gru"
        rcfg[m]["rnn_hidden_dim"] = 16
    runner = OnPolicyRunner(small_env(), rcfg, log_dir=None, device="cpu")
    runner.learn(2)


def test_b200_cfg_rejects_unknown_keys():
    from tt_rsl_rl_b200.algorithms.ppo import resolve_b200_cfg

    assert resolve_b200_cfg({"graphs": False})["graphs"] is False
    with pytest.raises(ValueError):
        resolve_b200_cfg({"nope": 1})


def test_b200_cfg_value_checks_and_exchange_policy():
    from tt_rsl_rl_b200.algorithms.ppo import resolve_b200_cfg, use_two_shot

    cfg = resolve_b200_cfg(None)
    assert cfg["exchange"] == "auto" and cfg["rnn_fused_step"] == "auto"
    for key, bad in (("exchange", "three_shot"), ("rnn_fused_step", "yes")):
        with pytest.raises(ValueError):
            resolve_b200_cfg({key: bad})
    for v in (True, False, "auto"):
        assert resolve_b200_cfg({"rnn_fused_step": v})["rnn_fused_step"] == v
    # "auto" exchanges in one shot (measured faster at the benchmark's size); two-shot only when asked, on 2+ ranks
    assert not any(use_two_shot(resolve_b200_cfg({"exchange": m}), w) for m in ("auto", "one_shot") for w in (1, 2, 8))
    assert use_two_shot(resolve_b200_cfg({"exchange": "two_shot"}), 2)
    assert not use_two_shot(resolve_b200_cfg({"exchange": "two_shot"}), 1)


# ---- data parallel over gloo (two CPU ranks) ------------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world, port, out_dir, reduce):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    import sys

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from helpers import ppo_cfg as cfg_fn
    from helpers import small_env as env_fn

    from tt_rsl_rl_b200.runners import OnPolicyRunner

    torch.manual_seed(rank)
    runner = OnPolicyRunner(env_fn(seed=rank), cfg_fn(), log_dir=None, device="cpu")
    if not reduce:
        runner.alg.reduce_parameters = lambda: None
    runner.learn(2)
    torch.save({k: v for k, v in runner.alg.actor.state_dict().items()}, os.path.join(out_dir, f"r{rank}.pt"))
    torch.distributed.destroy_process_group()


@pytest.mark.parametrize("reduce", [True, False])
def test_gloo_replicas_stay_identical_only_with_reduction(reduce):
    out = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_dp_worker, args=(2, _free_port(), out, reduce), nprocs=2, join=True)
    a = torch.load(os.path.join(out, "r0.pt"))
    b = torch.load(os.path.join(out, "r1.pt"))
    same = all(torch.equal(a[k], b[k]) for k in a)
    assert same == reduce


def _replica_worker(rank, world, port, out_dir, reduce):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    import sys

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from helpers import ppo_cfg as cfg_fn
    from helpers import small_env as env_fn

    from tt_rsl_rl_b200.parallel import ReplicaDivergenceError
    from tt_rsl_rl_b200.runners import OnPolicyRunner

    torch.manual_seed(rank)
    cfg = cfg_fn()
    cfg["algorithm"]["b200_cfg"] = {"replica_check_interval": 1}
    runner = OnPolicyRunner(env_fn(seed=rank), cfg, log_dir=None, device="cpu")
    if not reduce:
        runner.alg.reduce_parameters = lambda: None  # replicas drift apart after the first update
    try:
        runner.learn(2)
        result = "ok"
    except ReplicaDivergenceError as e:
        result = f"diverged: {e}"
    with open(os.path.join(out_dir, f"r{rank}"), "w") as f:
        f.write(result)
    torch.distributed.destroy_process_group()


@pytest.mark.parametrize("reduce", [True, False])
def test_replica_check_detects_divergence_on_every_rank(reduce):
    out = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_replica_worker, args=(2, _free_port(), out, reduce), nprocs=2, join=True)
    res = [open(os.path.join(out, f"r{r}")).read() for r in range(2)]
    if reduce:
        assert res == ["ok", "ok"], res
    else:
        assert all(r.startswith("diverged") and "after update 1" in r for r in res), res


# ---- host-side failure detection ---------------------------------------------------------------------------------------
def _wd_worker(rank, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    from tt_rsl_rl_b200.parallel import CommTimeoutError
    from tt_rsl_rl_b200.parallel.watchdog import RankWatchdog

    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=30))
    wd = RankWatchdog(store, rank, 2, timeout_s=1.5)
    wd.beat(0)
    wd.check(0)
    if rank == 1:
        # rank 1 fails between iterations: it never publishes iteration 1
        open(os.path.join(out_dir, "r1_exit"), "w").close()
        return
    wd.beat(1)
    import time

    t0 = time.monotonic()
    try:
        wd.check(1)
        result = "no-error"
    except CommTimeoutError as e:
        result = f"timeout {time.monotonic() - t0:.2f} {e}"
    with open(os.path.join(out_dir, "r0"), "w") as f:
        f.write(result)


def test_watchdog_reports_a_rank_that_left():
    out = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_wd_worker, args=(_free_port(), out), nprocs=2, join=True)
    res = open(os.path.join(out, "r0")).read()
    assert res.startswith("timeout"), res
    assert "[1]" in res
    assert float(res.split()[1]) < 5.0


def test_parity_report_metrics():
    from tt_rsl_rl_b200.testing import Tol, assert_parity, compare

    e = torch.linspace(-1, 1, 1001)
    rep = compare(e.clone(), e)
    assert rep.ok and rep.rel_fro == 0 and rep.max_ulp == 0 and rep.pcc == pytest.approx(1.0)
    a = e.clone()
    a[500] += 0.5  # one bad element
    rep = compare(a, e, Tol(rel_fro=1e-3))
    assert not rep.ok and rep.worst_index == (500,) and rep.max_abs == pytest.approx(0.5)
    nxt = torch.nextafter(e, torch.full_like(e, 2.0))
    assert compare(nxt, e).max_ulp == 1
    bf = e.to(torch.bfloat16).float()
    assert_parity(bf, e, "gemm_bf16", "bf16 rounding is within the bf16 GEMM tolerance")
    with pytest.raises(AssertionError):
        assert_parity(bf, e, "fp64_reduced", "but not within the fp64 one")


@pytest.mark.parametrize("rnn_type", ["gru", "lstm"])
def test_recurrent_minibatches_equal_a_done_masked_scan(rnn_type):
    """Upstream's split-and-pad trajectory minibatches (re-run from the state stored at each trajectory start) compute
    the same outputs as a time scan over the whole rollout whose input state is zeroed after every done: the basis of
    the fused recurrent engine's layout."""
    from tt_rsl_rl_b200.modules import RNN
    from tt_rsl_rl_b200.utils.utils import split_and_pad_trajectories

    torch.manual_seed(0)
    T, N, D, H = 12, 7, 5, 8
    rnn = RNN(D, H, 1, rnn_type)
    obs = torch.randn(T, N, D)
    dones = (torch.rand(T, N) < 0.2).float()
    h0 = torch.randn(1, N, H)
    c0 = torch.randn(1, N, H)
    # scan with masked state
    h, c = h0.clone(), c0.clone()
    scan = []
    with torch.no_grad():
        for t in range(T):
            if rnn_type == "gru":
                out, h = rnn.rnn(obs[t : t + 1], h)
            else:
                out, (h, c) = rnn.rnn(obs[t : t + 1], (h, c))
            scan.append(out[0])
            keep = (1 - dones[t])[None, :, None]
            h, c = h * keep, c * keep
    scan = torch.stack(scan)
    # trajectories: start state = rollout-start state for those starting at t = 0, reset (zero) state after a done
    padded, masks = split_and_pad_trajectories(obs, dones.unsqueeze(-1))
    starts = torch.zeros(T, N, dtype=torch.bool)
    starts[0] = True
    starts[1:] = dones[:-1].bool()
    hs, cs = [], []
    for n in range(N):  # trajectories are ordered env by env, then in time
        for t in range(T):
            if starts[t, n]:
                hs.append(h0[0, n] if t == 0 else torch.zeros(H))
                cs.append(c0[0, n] if t == 0 else torch.zeros(H))
    hid = torch.stack(hs)[None]
    state = hid if rnn_type == "gru" else (hid, torch.stack(cs)[None])
    with torch.no_grad():
        batched = rnn(padded, masks, state)
    torch.testing.assert_close(batched, scan, rtol=1e-5, atol=1e-6)


def test_normaliser_distributed_combine_with_a_fake_all_reduce(monkeypatch):
    """The three-all-reduce combine (count, sum, spread around the global mean) equals the statistics of the union
    of the ranks' batches; a second rank is simulated inside a fake ``all_reduce``."""
    from tt_rsl_rl_b200.modules import EmpiricalNormalization

    torch.manual_seed(1)
    x = torch.randn(50, 4) * 2 + 1  # this rank
    y = torch.randn(70, 4) - 3  # the simulated peer
    calls = []
    gmean = {}

    def fake_all_reduce(t, op=None):
        k = len(calls)
        calls.append(k)
        if k == 0:
            t += len(y)
        elif k == 1:
            t += y.mean(0, keepdim=True) * len(y)
            gmean["v"] = t / (len(x) + len(y))
        else:
            t += len(y) * (y.var(0, unbiased=False, keepdim=True) + (y.mean(0, keepdim=True) - gmean["v"]).square())

    monkeypatch.setattr(torch.distributed, "is_initialized", lambda: True)
    monkeypatch.setattr(torch.distributed, "all_reduce", fake_all_reduce)
    norm = EmpiricalNormalization(4)
    norm.train()
    norm.update(x)
    u = torch.cat([x, y])
    assert len(calls) == 3 and int(norm.count) == 120
    torch.testing.assert_close(norm._mean.squeeze(0), u.mean(0), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(norm._var.squeeze(0), u.var(0, unbiased=False), rtol=1e-5, atol=1e-6)


# ---- N ranks vs 1 rank on the union minibatch ------------------------------------------------------------------------
def _union_data(seed, N, T, D, A):
    g = torch.Generator().manual_seed(seed)
    return {
        "obs": torch.randn(T, N, D, generator=g), "actions": torch.randn(T, N, A, generator=g),
        "values": torch.randn(T, N, 1, generator=g), "mean": 0.1 * torch.randn(T, N, A, generator=g),
        "returns": torch.randn(T, N, 1, generator=g), "advantages": torch.randn(T, N, 1, generator=g),
    }


def _union_mirror(env=None, obs=None, actions=None):
    """Two copies: the observation vector reversed with alternating signs, the actions negated."""
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    out_obs = out_act = None
    if obs is not None:
        x = obs["policy"]
        sign = torch.ones(x.shape[1])
        sign[1::2] = -1.0
        out_obs = TensorDict({"policy": torch.cat([x, x.flip(1) * sign])}, batch_size=[2 * x.shape[0]])
    if actions is not None:
        out_act = torch.cat([actions, -actions])
    return out_obs, out_act


def _union_extensions(variant, D):
    if variant == "rnd":
        return {"rnd_cfg": {"num_states": D, "obs_groups": {"rnd_state": ["policy"]}, "num_outputs": 4,
                            "predictor_hidden_dims": [16], "target_hidden_dims": [16], "weight": 1.0,
                            "state_normalization": True}}
    if variant == "symmetry":
        return {"symmetry_cfg": {"env": None, "data_augmentation_func": _union_mirror, "use_data_augmentation": True,
                                 "use_mirror_loss": True, "mirror_loss_coeff": 0.5}}
    return {}


def _union_alg(data, multi_gpu_cfg=None, variant="plain"):
    from tt_rsl_rl_b200.algorithms import PPO
    from tt_rsl_rl_b200.models import MLPModel
    from tt_rsl_rl_b200.storage import RolloutStorage
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    T, N, D = data["obs"].shape
    A = data["actions"].shape[2]
    template = TensorDict({"policy": data["obs"][0]}, batch_size=[N])
    groups = {"actor": ["policy"], "critic": ["policy"]}
    torch.manual_seed(0)  # identical initial models everywhere
    actor = MLPModel(template, groups, "actor", A, hidden_dims=[32, 32], obs_normalization=True,
                     distribution_cfg={"class_name": "GaussianDistribution", "init_std": 1.0})
    critic = MLPModel(template, groups, "critic", 1, hidden_dims=[32, 32], obs_normalization=True)
    st = RolloutStorage("rl", N, T, template, [A], "cpu")
    dist = torch.distributions.Normal(data["mean"], torch.ones_like(data["mean"]))
    logp = dist.log_prob(data["actions"]).sum(-1, keepdim=True)
    for t in range(T):
        tr = RolloutStorage.Transition()
        tr.observations = TensorDict({"policy": data["obs"][t]}, batch_size=[N])
        tr.actions, tr.values, tr.actions_log_prob = data["actions"][t], data["values"][t], logp[t]
        tr.rewards, tr.dones = torch.zeros(N), torch.zeros(N)
        tr.distribution_params = (data["mean"][t], torch.ones(N, A))
        st.add_transition(tr)
    st.returns.copy_(data["returns"])
    st.advantages.copy_(data["advantages"])
    return PPO(actor, critic, st, num_learning_epochs=1, num_mini_batches=1, device="cpu",
               multi_gpu_cfg=multi_gpu_cfg, b200_cfg={"engine": "torch"}, **_union_extensions(variant, D))


def _models_of(alg):
    models = {"actor": alg.actor, "critic": alg.critic}
    if alg.rnd is not None:
        models["rnd_predictor"] = alg.rnd.predictor
        models["rnd_state_normalizer"] = alg.rnd.state_normalizer
    return models


def _union_worker(rank, world, port, out_dir, variant):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    alg = _union_alg(_union_data(10 + rank, 64, 6, 5, 3), {"global_rank": rank, "local_rank": rank,
                                                            "world_size": world}, variant)
    losses = alg.update()
    torch.save({**{k: m.state_dict() for k, m in _models_of(alg).items()}, "lr": alg.learning_rate,
                "losses": losses}, os.path.join(out_dir, f"r{rank}.pt"))
    torch.distributed.destroy_process_group()


@pytest.mark.parametrize("variant", ["plain", "rnd", "symmetry"])
def test_two_ranks_equal_one_rank_on_the_union_minibatch(variant):
    out = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_union_worker, args=(2, _free_port(), out, variant), nprocs=2, join=True)
    parts = [_union_data(10 + r, 64, 6, 5, 3) for r in range(2)]
    union = {k: torch.cat([parts[0][k], parts[1][k]], dim=1) for k in parts[0]}
    alg = _union_alg(union, variant=variant)
    alg.update()
    for r in range(2):
        got = torch.load(os.path.join(out, f"r{r}.pt"))
        assert got["lr"] == pytest.approx(alg.learning_rate, rel=1e-6)
        for name, model in _models_of(alg).items():
            for k, v in model.state_dict().items():
                torch.testing.assert_close(got[name][k], v, rtol=1e-5, atol=1e-6, msg=f"rank {r} {name}.{k}")


# ---- distillation: N ranks vs 1 rank on the union batch -------------------------------------------------------------
def _distill_union_data(seed, N, T, D, A):
    g = torch.Generator().manual_seed(seed)
    return {"obs": torch.randn(T, N, D, generator=g), "teacher": torch.randn(T, N, A, generator=g)}


def _distill_union_alg(data, multi_gpu_cfg=None):
    from tt_rsl_rl_b200.algorithms import Distillation
    from tt_rsl_rl_b200.models import MLPModel
    from tt_rsl_rl_b200.storage import RolloutStorage
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    T, N, D = data["obs"].shape
    A = data["teacher"].shape[2]
    template = TensorDict({"policy": data["obs"][0]}, batch_size=[N])
    groups = {"student": ["policy"], "teacher": ["policy"]}
    torch.manual_seed(0)
    student = MLPModel(template, groups, "student", A, hidden_dims=[32, 32], obs_normalization=True,
                       distribution_cfg={"class_name": "GaussianDistribution", "init_std": 1.0})
    teacher = MLPModel(template, groups, "teacher", A, hidden_dims=[32, 32])
    st = RolloutStorage("distillation", N, T, template, [A], "cpu")
    for t in range(T):
        tr = RolloutStorage.Transition()
        tr.observations = TensorDict({"policy": data["obs"][t]}, batch_size=[N])
        tr.actions = torch.zeros(N, A)
        tr.privileged_actions = data["teacher"][t]
        tr.rewards, tr.dones = torch.zeros(N), torch.zeros(N)
        st.add_transition(tr)
    return Distillation(student, teacher, st, num_learning_epochs=2, gradient_length=3, max_grad_norm=1.0,
                        device="cpu", multi_gpu_cfg=multi_gpu_cfg, b200_cfg={"engine": "torch"})


def _distill_union_worker(rank, world, port, out_dir):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    alg = _distill_union_alg(_distill_union_data(20 + rank, 32, 6, 5, 3),
                             {"global_rank": rank, "local_rank": rank, "world_size": world})
    alg.update()
    torch.save(alg.student.state_dict(), os.path.join(out_dir, f"d{rank}.pt"))
    torch.distributed.destroy_process_group()


def test_distillation_two_ranks_equal_one_rank_on_the_union_batch():
    """Rank-averaged gradients of equal-sized local batches equal the gradient of the union batch, and the student
    normaliser's global statistics equal the union's (the reference plugin's distillation equivalence test has the
    same design: ``rsl_rl_tt/testing/distill_equiv.py:32-81``)."""
    out = tempfile.mkdtemp()
    torch.multiprocessing.spawn(_distill_union_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    parts = [_distill_union_data(20 + r, 32, 6, 5, 3) for r in range(2)]
    union = {k: torch.cat([parts[0][k], parts[1][k]], dim=1) for k in parts[0]}
    alg = _distill_union_alg(union)
    alg.update()
    for r in range(2):
        got = torch.load(os.path.join(out, f"d{r}.pt"))
        for k, v in alg.student.state_dict().items():
            torch.testing.assert_close(got[k], v, rtol=1e-5, atol=1e-6, msg=f"rank {r} student.{k}")


# ---- host-side GEMM planning of the fused engines (no device work) --------------------------------------------------------
@pytest.mark.parametrize("in_dim,hidden,A,rows", [(96, [512, 256, 128], 29, 98304), (99, [1024, 1024, 512], 1, 4096),
                                                   (5, [32], 3, 100)])
def test_mlp_plan_buffers_and_reduction_segments(in_dim, hidden, A, rows):
    """Buffers of the per-MLP GEMM plan obey the 16-byte row-pitch rule of TMA, the split-K factor fills the GPU once
    without exceeding the k-blocks, and every weight and bias has a partial-sum segment of the right size."""
    from tt_rsl_rl_b200.engine.mlp_plan import MLPPlan, pad8, wgrad_splits
    from tt_rsl_rl_b200.modules.mlp import MLP

    mlp = MLP(in_dim, A, hidden, "elu")
    sm = 148
    plan = MLPPlan(mlp, in_dim, rows_roll=rows // 4, rows_train=rows, device=torch.device("cpu"), sm_count=sm)
    bf16 = [plan.x_roll, plan.x_train, plan.d_head, *plan.h_roll, *plan.h_train, *plan.dz, *plan.w_bf16]
    assert all(t.dtype == torch.bfloat16 and t.shape[-1] % 8 == 0 for t in bf16)  # 16-byte pitches
    # fp32 head outputs: pitch rounded up to whole 32-column chunks of the GEMM epilogue
    assert plan.out_roll.shape[1] == plan.out_train.shape[1] == plan.out_pitch == (A + 31) // 32 * 32
    assert plan.widths == [in_dim, *hidden, A]
    for lin, s, part in zip(plan.linears, plan.splits, plan.wgrad_partial):
        kb = (rows + 63) // 64
        assert 1 <= s <= kb and part.shape == (s, lin.out_features, lin.in_features)
        assert s == wgrad_splits(lin.out_features, lin.in_features, rows, sm)
    head = torch.zeros(7, A)
    segs = plan.reduce_segments(head, 7)
    for l, lin in enumerate(plan.linears):
        buf, parts, n = segs[id(lin.weight)]
        assert n == lin.weight.numel() and buf.numel() == parts * n
        buf, parts, n = segs[id(lin.bias)]
        assert n == lin.bias.numel() and buf.numel() == parts * n
        if l == plan.L - 1:
            assert buf is head
    assert len(segs) == 2 * plan.L
    assert pad8(1) == 8 and pad8(8) == 8 and pad8(29) == 32


def test_which_configurations_the_fused_engines_take():
    """The engines' own checks (host-side, no device): what runs fused and why the rest stays on the PyTorch path."""
    from tt_rsl_rl_b200.engine import PPOEngine, RecurrentPPOEngine
    from tt_rsl_rl_b200.models import CNNModel, MLPModel, RNNModel
    from tt_rsl_rl_b200.utils.tensordict import TensorDict

    obs = TensorDict({"policy": torch.zeros(2, 8), "image": torch.zeros(2, 1, 8, 8)}, batch_size=[2])
    g = {"actor": ["policy"], "critic": ["policy"]}
    gauss = {"class_name": "GaussianDistribution"}

    def mlp(role, out, act="elu", dist=None, hidden=(32, 32)):
        return MLPModel(obs, g, role, out, hidden_dims=list(hidden), activation=act, distribution_cfg=dist)

    ok = PPOEngine.supports_models(mlp("actor", 3, dist=gauss), mlp("critic", 1), {})
    assert ok is None
    hetero = {"class_name": "HeteroscedasticGaussianDistribution"}
    assert PPOEngine.supports_models(mlp("actor", 3, dist=hetero), mlp("critic", 1), {}) is None
    assert "ELU" in PPOEngine.supports_models(mlp("actor", 3, act="relu", dist=gauss), mlp("critic", 1), {})
    assert "Gaussian" in PPOEngine.supports_models(mlp("actor", 3, dist={"class_name": "BetaDistribution"}),
                                                   mlp("critic", 1), {})
    assert "32 actions" in PPOEngine.supports_models(mlp("actor", 40, dist=gauss), mlp("critic", 1), {})
    assert "Adam" in PPOEngine.supports_models(mlp("actor", 3, dist=gauss), mlp("critic", 1), {"optimizer": "sgd"})
    cnn_g = {"actor": ["policy", "image"], "critic": ["policy", "image"]}
    cnn = CNNModel(obs, cnn_g, "actor", 3, hidden_dims=[16], distribution_cfg=gauss,
                   cnn_cfg={"output_channels": [4], "kernel_size": 3})
    assert "CNN" in PPOEngine.supports_models(cnn, mlp("critic", 1), {})

    def rnn(role, out, dist=None, rnn_type="gru", hidden=32, layers=1):
        return RNNModel(obs, g, role, out, hidden_dims=[16], distribution_cfg=dist, rnn_type=rnn_type,
                        rnn_hidden_dim=hidden, rnn_num_layers=layers)

    assert RecurrentPPOEngine.supports_models(rnn("actor", 3, gauss), rnn("critic", 1), {}) is None
    assert RecurrentPPOEngine.supports_models(rnn("actor", 3, gauss, "lstm"), rnn("critic", 1, None, "lstm"), {}) is None
    assert "single-layer" in RecurrentPPOEngine.supports_models(rnn("actor", 3, gauss, layers=2), rnn("critic", 1), {})
    assert "multiple of 32" in RecurrentPPOEngine.supports_models(rnn("actor", 3, gauss, hidden=20),
                                                                  rnn("critic", 1), {})
    # RND with recurrent models runs fused (ELU networks only, as on the MLP engine)
    assert RecurrentPPOEngine.supports_models(rnn("actor", 3, gauss), rnn("critic", 1), {"rnd_cfg": {}}) is None
    assert "RND" in RecurrentPPOEngine.supports_models(rnn("actor", 3, gauss), rnn("critic", 1),
                                                       {"rnd_cfg": {"activation": "relu"}})
    assert "not fused" in PPOEngine.supports_models(rnn("actor", 3, gauss), rnn("critic", 1), {})

    # distillation: MLP or recurrent students, MLP or recurrent teachers
    from types import SimpleNamespace

    from tt_rsl_rl_b200.engine import DistillationEngine, RecurrentDistillationEngine

    gd = {"student": ["policy"], "teacher": ["policy"]}
    s_rnn = RNNModel(obs, gd, "student", 3, hidden_dims=[16], distribution_cfg=gauss, rnn_type="lstm",
                     rnn_hidden_dim=32)
    t_rnn = RNNModel(obs, gd, "teacher", 3, hidden_dims=[16], rnn_type="gru", rnn_hidden_dim=64)
    t_mlp = MLPModel(obs, gd, "teacher", 3, hidden_dims=[32])
    alg = SimpleNamespace(student=s_rnn, teacher=t_rnn, loss_type="mse", optimizer_name="adam")
    assert RecurrentDistillationEngine.unsupported_reason(alg) is None
    alg.teacher = t_mlp
    assert RecurrentDistillationEngine.unsupported_reason(alg) is None
    assert "not fused" in DistillationEngine.unsupported_reason(alg)  # the MLP engine takes MLP students only
    alg.student = MLPModel(obs, gd, "student", 3, hidden_dims=[32], distribution_cfg=gauss)
    assert DistillationEngine.unsupported_reason(alg) is None
    alg.teacher = t_rnn
    assert DistillationEngine.unsupported_reason(alg) is None
    alg.teacher = RNNModel(obs, gd, "teacher", 3, hidden_dims=[16], rnn_type="gru", rnn_hidden_dim=20)
    assert "multiple of 32" in DistillationEngine.unsupported_reason(alg)
