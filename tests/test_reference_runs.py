"""Reference-run harness: mirror functions of the test environments and the signed-permutation probe, run specs and
config builders on both implementations, the CSV writer, and the golden acceptance rule."""

import math
import os

import pytest
import torch

from tt_rsl_rl_b200.env import make_env
from tt_rsl_rl_b200.extensions import Symmetry
from tt_rsl_rl_b200.testing import golden
from tt_rsl_rl_b200.testing import reference as R
from tt_rsl_rl_b200.testing import symmetry as S


def _probe(env_name, func):
    env = make_env(env_name, 4, seed=0)
    sym = Symmetry(env, func, use_data_augmentation=True)
    return sym.probe_signed_permutations(env.get_observations(), env.num_actions)


@pytest.mark.parametrize("env_name,func,K", [
    ("cartpole", S.cartpole_mirror, 2), ("cartpole_po", S.cartpole_mirror, 2), ("pendulum", S.pendulum_mirror, 2),
    ("tracking12", S.tracking12_sign_mirror, 2), ("tracking12", S.tracking12_dihedral_mirror, 4),
])
def test_mirrors_are_signed_permutations_and_symmetries(env_name, func, K):
    maps = _probe(env_name, func)
    assert maps is not None
    obs_maps, act_maps = maps
    assert act_maps[0].shape[0] == K and all(p.shape[0] == K for p, _ in obs_maps.values())
    # a true symmetry: mirrored states evolve into mirrored states with equal rewards
    a, b = make_env(env_name, 8, seed=2), make_env(env_name, 8, seed=2)
    if env_name == "tracking12":
        for k in ("p", "v", "a_prev", "amp", "omega", "phase"):
            getattr(b, k).copy_(getattr(a, k))
        b.p.neg_(), b.v.neg_(), b.a_prev.neg_()
        b.phase.add_(math.pi)
    elif env_name == "pendulum":
        b.th, b.thd = -a.th.clone(), -a.thd.clone()
    else:
        b.s = -a.s.clone()
    acts = torch.randn(8, a.num_actions) * 0.3
    for _ in range(5):
        oa, ra, _, _ = a.step(acts)
        ob, rb, _, _ = b.step(-acts)
        mirrored, _ = S.MIRRORS[env_name](obs=oa)
        for g in oa.keys():
            torch.testing.assert_close(ob[g], mirrored[g][8:], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(ra, rb, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("func", [S.tracking12_affine_mirror, S.tracking12_mixing_mirror, S.tracking12_cubic_mirror])
def test_probe_refuses_maps_that_are_not_signed_permutations(func):
    assert _probe("tracking12", func) is None


def test_config_builders():
    spec = R.with_symmetry("tracking12", R.with_rnd("tracking12", R.SPECS["tracking12"]))
    cfg = R.train_cfg("tracking12", spec)
    alg = cfg["algorithm"]
    assert alg["rnd_cfg"]["weight"] == R.RND_WEIGHT["tracking12"]
    assert alg["symmetry_cfg"]["data_augmentation_func"].endswith(":tracking12_sign_mirror")
    assert cfg["obs_groups"] == {"actor": ["policy"], "critic": ["policy", "privileged"]}
    rnn = R.train_cfg("cartpole", R.with_rnn(R.SPECS["cartpole"], "lstm", critic=False))
    assert rnn["actor"]["class_name"] == "RNNModel" and rnn["actor"]["rnn_type"] == "lstm"
    assert rnn["critic"]["class_name"] == "MLPModel"
    t = R.teacher_train_cfg("tracking12")
    assert t["obs_groups"]["actor"] == ["policy", "privileged"]
    d = R.distill_cfg("tracking12")
    assert d["obs_groups"]["student"] == ["policy"] and d["algorithm"]["class_name"] == "Distillation"
    with pytest.raises(ValueError):
        R.build_runner("cartpole", 0, impl="upstream", device="cuda:0")


def _small(spec, **kw):
    import dataclasses

    return dataclasses.replace(spec, num_envs=64, num_steps=8, **kw)


@pytest.mark.parametrize("impl", ["b200", "upstream"])
@pytest.mark.parametrize("variant", ["plain", "rnd_symmetry", "gru"])
def test_runs_of_both_implementations_log_the_same_columns(ref, tmp_path, impl, variant):
    env_name = "cartpole_po" if variant == "gru" else "tracking12"
    spec = _small(R.SPECS[env_name])
    if variant == "rnd_symmetry":
        spec = R.with_symmetry(env_name, R.with_rnd(env_name, spec))
    out = R.train(env_name, 0, str(tmp_path), impl=impl, iterations=3, spec=spec)
    assert out["iterations"] == 3
    rows = golden.read_curve(tmp_path / "metrics.csv")
    assert [r["iteration"] for r in rows] == [0, 1, 2]
    assert all(math.isfinite(r["Loss/value"]) for r in rows)
    if variant == "rnd_symmetry":
        assert "Loss/rnd" in rows[0] and "Loss/symmetry" in rows[0]


@pytest.mark.parametrize("impl", ["b200", "upstream"])
def test_teacher_checkpoint_and_distillation(ref, tmp_path, impl):
    ckpt = R.make_teacher_checkpoint("tracking12", str(tmp_path / "teacher.pt"), iterations=2, num_envs=64,
                                     impl=impl)
    assert os.path.exists(ckpt)
    out = R.train_distillation("tracking12", 0, str(tmp_path / "d"), ckpt, impl=impl, iterations=2)
    assert out["iterations"] == 2
    rows = golden.read_curve(tmp_path / "d" / "metrics.csv")
    assert len(rows) == 2 and "Loss/behavior" in rows[0]


def test_csv_writer_keeps_late_columns(tmp_path):
    from tt_rsl_rl_b200.utils.log_writer import CsvLogWriter

    w = CsvLogWriter(str(tmp_path))
    w.add_scalar("Loss/value", 1.0, 0)
    w.add_scalar("Train/mean_reward/time", 5.0, 17)  # time-indexed: skipped
    w.add_scalar("Loss/value", 2.0, 1)
    w.add_scalar("Train/mean_reward", 3.0, 1)
    w.stop()
    rows = golden.read_curve(tmp_path / "metrics.csv")
    assert [r["iteration"] for r in rows] == [0, 1]
    assert rows[0]["Train/mean_reward"] is None and rows[1]["Train/mean_reward"] == 3.0


def test_golden_rule(tmp_path):
    rows = [{"iteration": i, "Train/mean_reward": float(i)} for i in range(30)]
    assert golden.final_reward(rows) == pytest.approx(sum(range(20, 30)) / 10)
    assert math.isnan(golden.final_reward([{"iteration": 0, "Train/mean_reward": None}]))
    summary = {"envs": {"x": {"final_reward_mean": 100.0, "final_reward_std": 2.0}}}
    assert golden.threshold(100.0, 2.0) == 95.0 and golden.threshold(-10.0, 2.0) == -12.0
    assert golden.verdict("x", [96.0, 95.0], summary=summary)["passes"]
    assert not golden.verdict("x", [94.0, 95.0], summary=summary)["passes"]
    assert not golden.verdict("x", [float("nan"), 200.0], summary=summary)["passes"]
    assert not golden.verdict("x", [99.0], curves_finite=False, summary=summary)["passes"]
    golden.write_curve(tmp_path / "c.csv", rows)
    assert golden.read_curve(tmp_path / "c.csv")[5]["Train/mean_reward"] == 5.0


def test_committed_golden_curves_are_consistent():
    summary = golden.load_summary()
    assert set(summary["envs"]) >= {"cartpole", "pendulum", "tracking12", "cartpole_po"}
    for env_name, ref in summary["envs"].items():
        assert tuple(ref["seeds"]) == golden.seeds_for(env_name)
        finals = [golden.final_reward(golden.read_curve(golden.GOLDEN_DIR / env_name / f"seed{s}.csv"))
                  for s in ref["seeds"]]
        assert finals == pytest.approx(ref["final_rewards"])


def test_this_framework_passes_the_golden_rule_on_cartpole():
    """One seed of the cart-pole spec on the CPU path against the upstream golden curves."""
    (res,) = golden.check(["cartpole"], seeds=(0,))
    assert res["all_finite"]
    assert res["mean"] >= res["threshold"], res


def test_cpu_path_reproduces_the_upstream_curve_exactly():
    """Same seed, same environment: the PyTorch path logs the same numbers as upstream rsl_rl did for the golden
    curve (the first 10 iterations of cart-pole seed 0), not just a statistically equivalent curve."""
    import tempfile

    threads = torch.get_num_threads()
    torch.set_num_threads(2)  # the thread count of the recording
    try:
        with tempfile.TemporaryDirectory() as tmp:
            R.train("cartpole", 0, tmp, iterations=10)
            ours = golden.read_curve(os.path.join(tmp, "metrics.csv"))
    finally:
        torch.set_num_threads(threads)
    gold = golden.read_curve(golden.GOLDEN_DIR / "cartpole" / "seed0.csv")[:10]
    for g, o in zip(gold, ours):
        for k, v in g.items():
            if v is not None:
                assert o[k] == v, (g["iteration"], k, v, o[k])


def test_episode_extras_are_logged_every_iteration_like_upstream(ref, tmp_path):
    """``extras["log"]`` means (here the cart-pole's pole angle) appear in every iteration's log with upstream's
    values."""
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        rows = {}
        for impl in ("b200", "upstream"):
            R.train("cartpole", 0, str(tmp_path / impl), impl=impl, iterations=3)
            rows[impl] = golden.read_curve(tmp_path / impl / "metrics.csv")
    finally:
        torch.set_num_threads(threads)
    ours, theirs = ([r.get("Episode/pole_angle") for r in rows[k]] for k in ("b200", "upstream"))
    assert len(ours) == 3 and all(v is not None for v in ours)
    assert ours == theirs


@pytest.mark.parametrize("variant", ["rnd_symmetry", "gru", "lstm", "hetero", "per_minibatch_fixed_lr", "beta",
                                     "log_std_unclipped", "cnn", "mixed_precision", "mirror_loss_only",
                                     "rnd_linear_schedule", "sgd", "rmsprop", "adamw"])
def test_every_logged_scalar_equals_upstream(ref, tmp_path, variant):
    """Same seeds, same thread count: every logged column except timings is equal to upstream's, iteration by
    iteration."""
    import dataclasses

    small = dict(num_envs=64, num_steps=8)
    if variant == "rnd_symmetry":
        env_name = "tracking12"
        spec = R.with_symmetry(env_name, R.with_rnd(env_name, dataclasses.replace(R.SPECS[env_name], **small)))
    elif variant == "gru":
        env_name, spec = "cartpole_po", dataclasses.replace(R.SPECS["cartpole_po"], **small)
    elif variant == "lstm":
        env_name = "tracking12"
        spec = R.with_rnn(dataclasses.replace(R.SPECS[env_name], **small), "lstm", 32)
    elif variant == "hetero":
        env_name = "pendulum"
        spec = dataclasses.replace(R.SPECS[env_name], distribution="HeteroscedasticGaussianDistribution", **small)
    elif variant == "per_minibatch_fixed_lr":
        env_name = "cartpole"
        alg = {**R.SPECS[env_name].algorithm, "normalize_advantage_per_mini_batch": True, "schedule": "fixed"}
        spec = dataclasses.replace(R.SPECS[env_name], algorithm=alg, **small)
    elif variant == "cnn":
        env_name = "cartpole_image"
        cnn = {"class_name": "CNNModel", "cnn_cfg": {"output_channels": [4, 8], "kernel_size": 3, "stride": [1, 2],
                                                     "norm": "batch", "activation": "elu"}}
        spec = dataclasses.replace(R.SPECS["cartpole"], hidden=(32,), model=cnn, **small)
    elif variant == "mirror_loss_only":
        env_name = "tracking12"
        spec = R.with_symmetry(env_name, dataclasses.replace(R.SPECS[env_name], **small), data_augmentation=False)
    elif variant == "rnd_linear_schedule":
        env_name = "tracking12"
        spec = R.with_rnd(env_name, dataclasses.replace(R.SPECS[env_name], **small))
        rnd = {**spec.algorithm["rnd_cfg"], "weight_schedule": {"mode": "linear", "initial_step": 4,
                                                                "final_step": 20, "final_value": 0.0}}
        spec = dataclasses.replace(spec, algorithm={**spec.algorithm, "rnd_cfg": rnd})
    elif variant in ("sgd", "rmsprop", "adamw"):
        env_name = "cartpole"
        alg = {**R.SPECS[env_name].algorithm, "optimizer": variant}
        spec = dataclasses.replace(R.SPECS[env_name], algorithm=alg, **small)
    elif variant == "mixed_precision":
        env_name = "tracking12"
        alg = {**R.SPECS[env_name].algorithm, "use_mixed_precision": True}
        spec = dataclasses.replace(R.SPECS[env_name], algorithm=alg, **small)
    elif variant == "beta":
        env_name = "pendulum"
        spec = dataclasses.replace(R.SPECS[env_name], distribution="BetaDistribution", **small)
    else:
        env_name = "tracking12"
        alg = {**R.SPECS[env_name].algorithm, "use_clipped_value_loss": False, "entropy_coef": 0.01}
        spec = dataclasses.replace(R.SPECS[env_name], algorithm=alg, model={"distribution_cfg": {
            "class_name": "GaussianDistribution", "init_std": 1.0, "std_type": "log"}}, critic_model={}, **small)
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        rows = {}
        for impl in ("b200", "upstream"):
            R.train(env_name, 0, str(tmp_path / impl), impl=impl, iterations=3, spec=spec)
            rows[impl] = golden.read_curve(tmp_path / impl / "metrics.csv")
    finally:
        torch.set_num_threads(threads)
    cols = {k for r in rows["upstream"] for k in r} | {k for r in rows["b200"] for k in r}
    for c in sorted(cols):
        if c.startswith("Perf/") or c == "wall_s":
            continue
        ours, theirs = [r.get(c) for r in rows["b200"]], [r.get(c) for r in rows["upstream"]]
        assert ours == theirs, c


def _equal_state(a, b, where):
    if isinstance(b, dict):
        assert sorted(a, key=str) == sorted(b, key=str), where
        for k in b:
            _equal_state(a[k], b[k], f"{where}.{k}")
    elif isinstance(b, (list, tuple)):
        assert len(a) == len(b), where
        for i, (x, y) in enumerate(zip(a, b)):
            _equal_state(x, y, f"{where}[{i}]")
    elif isinstance(b, torch.Tensor) or isinstance(a, torch.Tensor):
        assert torch.equal(torch.as_tensor(a), torch.as_tensor(b)), where
    else:
        assert a == b, where


@pytest.mark.parametrize("variant", ["plain", "rnd_symmetry", "gru", "lstm", "cnn", "hetero_log_std", "beta"])
def test_checkpoints_after_training_equal_upstream(ref, tmp_path, variant):
    """Three iterations from the same seed: the saved checkpoints (models, normalisers, Adam state, RND networks and
    counters, iteration) of this framework and of upstream are equal tensor by tensor."""
    import dataclasses

    env_name = {"gru": "cartpole_po", "cnn": "cartpole_image", "beta": "pendulum"}.get(variant, "tracking12")
    base = R.SPECS["cartpole"] if env_name == "cartpole_image" else R.SPECS[env_name]
    spec = dataclasses.replace(base, num_envs=64, num_steps=8)
    if variant == "rnd_symmetry":
        spec = R.with_symmetry(env_name, R.with_rnd(env_name, spec))
    elif variant == "lstm":
        spec = R.with_rnn(spec, "lstm", 32)
    elif variant == "cnn":
        spec = dataclasses.replace(spec, hidden=(32,), model={"class_name": "CNNModel", "cnn_cfg": {
            "output_channels": [4], "kernel_size": 3, "norm": "batch", "activation": "elu"}})
    elif variant == "hetero_log_std":
        spec = dataclasses.replace(spec, model={"distribution_cfg": {
            "class_name": "HeteroscedasticGaussianDistribution", "init_std": 1.0, "std_type": "log"}}, critic_model={})
    elif variant == "beta":
        spec = dataclasses.replace(spec, distribution="BetaDistribution")
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    saved = {}
    try:
        for impl in ("b200", "upstream"):
            runner, _, _ = R.build_runner(env_name, 0, None, spec, impl=impl)
            runner.learn(3, init_at_random_ep_len=True)
            runner.save(str(tmp_path / f"{impl}.pt"))
            saved[impl] = torch.load(tmp_path / f"{impl}.pt", weights_only=False)
    finally:
        torch.set_num_threads(threads)
    ours, theirs = saved["b200"], saved["upstream"]
    assert ours["iter"] == theirs["iter"] == 2
    assert sorted(ours) == sorted(theirs)
    for key in theirs:
        if key in ("actor_state_dict", "critic_state_dict", "rnd_state_dict"):
            assert list(ours[key]) == list(theirs[key]), key  # same names in the same order
        _equal_state(ours[key], theirs[key], key)


@pytest.mark.parametrize("loss_type,student", [("mse", None), ("huber", None), ("mse", "gru"), ("huber", "lstm")])
def test_distillation_logs_equal_upstream(ref, tmp_path, loss_type, student):
    """Distillation from the same teacher checkpoint: every logged scalar equals upstream's."""
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        ckpt = R.make_teacher_checkpoint("tracking12", str(tmp_path / "t.pt"), iterations=2, num_envs=64,
                                         impl="upstream")
        rows = {}
        for impl in ("b200", "upstream"):
            student_model = None if student is None else {"class_name": "RNNModel", "rnn_type": student,
                                                          "rnn_hidden_dim": 32}
            R.train_distillation("tracking12", 0, str(tmp_path / impl), ckpt, impl=impl, iterations=3,
                                 algorithm={"loss_type": loss_type}, student_model=student_model)
            rows[impl] = golden.read_curve(tmp_path / impl / "metrics.csv")
    finally:
        torch.set_num_threads(threads)
    for c in sorted({k for r in rows["upstream"] for k in r}):
        if c.startswith("Perf/") or c == "wall_s":
            continue
        ours, theirs = [r.get(c) for r in rows["b200"]], [r.get(c) for r in rows["upstream"]]
        assert ours == theirs, c


def test_tensorboard_runs_convert_and_compare(tmp_path):
    from torch.utils.tensorboard import SummaryWriter

    for seed, level in ((0, 100.0), (1, 104.0)):
        w = SummaryWriter(str(tmp_path / f"tb{seed}"))
        for it in range(20):
            w.add_scalar("Train/mean_reward", level * it / 19, it)
            w.add_scalar("Loss/value", 1.0 / (it + 1), it)
            w.add_scalar("Train/mean_reward/time", 0.0, 1000 + it)  # time-indexed duplicates are dropped
        w.close()
        assert golden.tb_to_csv(tmp_path / f"tb{seed}", tmp_path / f"ref{seed}.csv") == 20
    rows = golden.read_curve(tmp_path / "ref0.csv")
    assert rows[19]["Train/mean_reward"] == pytest.approx(100.0) and "Train/mean_reward/time" not in rows[0]
    good = [{"iteration": i, "Train/mean_reward": 100.0} for i in range(20)]
    bad = [{"iteration": i, "Train/mean_reward": 50.0} for i in range(20)]
    golden.write_curve(tmp_path / "good.csv", good)
    golden.write_curve(tmp_path / "bad.csv", bad)
    refs = [tmp_path / "ref0.csv", tmp_path / "ref1.csv"]
    assert golden.compare_runs(refs, [tmp_path / "good.csv"])["passes"]
    assert not golden.compare_runs(refs, [tmp_path / "bad.csv"])["passes"]
    assert golden.main(["compare", "--ref", *map(str, refs), "--run", str(tmp_path / "good.csv")]) == 0


def test_stability_measures():
    rise = [{"iteration": i, "Train/mean_reward": min(500.0, 50.0 * i)} for i in range(15)]
    s = golden.stability(rise)
    assert s["first_at_level"] == 10 and s["min_after"] == 500.0 and not s["collapsed"]
    dip = rise + [{"iteration": 15, "Train/mean_reward": 300.0}, {"iteration": 16, "Train/mean_reward": 500.0}]
    assert golden.stability(dip)["collapsed"]
    assert golden.stability([{"iteration": 0, "Train/mean_reward": 10.0}])["first_at_level"] is None


def test_distillation_checkpoints_after_training_equal_upstream(ref, tmp_path):
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    saved = {}
    try:
        ckpt = R.make_teacher_checkpoint("tracking12", str(tmp_path / "t.pt"), iterations=2, num_envs=64,
                                         impl="upstream")
        for impl in ("b200", "upstream"):
            runner, _, _ = R.build_distillation_runner("tracking12", 0, None, ckpt, impl=impl, num_envs=64,
                                                       student_model={"class_name": "RNNModel", "rnn_type": "gru",
                                                                      "rnn_hidden_dim": 32})
            runner.learn(3, init_at_random_ep_len=True)
            runner.save(str(tmp_path / f"{impl}.pt"))
            saved[impl] = torch.load(tmp_path / f"{impl}.pt", weights_only=False)
    finally:
        torch.set_num_threads(threads)
    assert sorted(saved["b200"]) == sorted(saved["upstream"])
    for key in saved["upstream"]:
        _equal_state(saved["b200"][key], saved["upstream"][key], key)


def test_resumed_training_equals_upstream(ref, tmp_path):
    """Save after two iterations, load into a fresh runner and train two more: iteration numbers, logged scalars and
    the final checkpoint equal upstream's doing the same."""
    import dataclasses

    spec = dataclasses.replace(R.SPECS["tracking12"], num_envs=64, num_steps=8)
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    out = {}
    try:
        for impl in ("b200", "upstream"):
            first, _, _ = R.build_runner("tracking12", 0, None, spec, impl=impl)
            first.learn(2, init_at_random_ep_len=True)
            first.save(str(tmp_path / f"{impl}_a.pt"))
            log_dir = str(tmp_path / impl)
            second, _, _ = R.build_runner("tracking12", 1, log_dir, spec, impl=impl)
            second.load(str(tmp_path / f"{impl}_a.pt"))
            second.learn(2)
            second.logger.writer.stop()
            out[impl] = (golden.read_curve(tmp_path / impl / "metrics.csv"),
                         torch.load(os.path.join(log_dir, "model_2.pt"), weights_only=False))
    finally:
        torch.set_num_threads(threads)
    (rows_o, ck_o), (rows_u, ck_u) = out["b200"], out["upstream"]
    assert [r["iteration"] for r in rows_o] == [r["iteration"] for r in rows_u] == [1, 2]
    for c in rows_u[0]:
        if not c.startswith("Perf/") and c != "wall_s":
            assert [r.get(c) for r in rows_o] == [r.get(c) for r in rows_u], c
    for key in ck_u:
        _equal_state(ck_o[key], ck_u[key], key)


PARITY_DRAWS = int(os.environ.get("RLB_PARITY_DRAWS", "6"))  # more draws for a longer sweep


@pytest.mark.parametrize("draw", range(PARITY_DRAWS))
def test_random_configurations_log_exactly_what_upstream_logs(ref, tmp_path, draw):
    """Randomly drawn algorithm settings (epochs, minibatches, clip, discounting, KL target or a fixed learning rate,
    gradient-norm limits, loss weights, network sizes, normalisation): every logged scalar equals upstream's."""
    import dataclasses
    import random

    rng = random.Random(1000 + draw)
    env_name = rng.choice(["cartpole", "pendulum", "tracking12"])
    schedule = rng.choice(["adaptive", "fixed"])
    alg = {**R.PPO_ALGORITHM,
           "num_learning_epochs": rng.randint(1, 4), "num_mini_batches": rng.choice([1, 2, 3, 4, 7]),
           "clip_param": rng.choice([0.1, 0.2, 0.3]), "gamma": rng.choice([0.9, 0.99, 0.999]),
           "lam": rng.choice([0.9, 0.95, 1.0]), "value_loss_coef": rng.choice([0.5, 1.0, 2.0]),
           "entropy_coef": rng.choice([0.0, 0.005, 0.02]), "learning_rate": rng.choice([3e-4, 1e-3, 3e-3]),
           "max_grad_norm": rng.choice([0.5, 1.0, 10.0]), "schedule": schedule,
           "desired_kl": rng.choice([0.005, 0.01, 0.02]) if schedule == "adaptive" else None,
           "use_clipped_value_loss": rng.choice([True, False]),
           "normalize_advantage_per_mini_batch": rng.choice([True, False])}
    hidden = tuple(rng.choice([16, 32, 64]) for _ in range(rng.randint(1, 3)))
    spec = dataclasses.replace(R.SPECS[env_name], num_envs=rng.choice([16, 48, 64]), num_steps=rng.choice([4, 8, 12]),
                               hidden=hidden, algorithm=alg, obs_normalization=rng.choice([True, False]),
                               init_std=rng.choice([0.5, 1.0]))
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        rows = {}
        for impl in ("b200", "upstream"):
            R.train(env_name, draw, str(tmp_path / impl), impl=impl, iterations=3, spec=spec)
            rows[impl] = golden.read_curve(tmp_path / impl / "metrics.csv")
    finally:
        torch.set_num_threads(threads)
    cols = {k for r in rows["upstream"] for k in r} | {k for r in rows["b200"] for k in r}
    for c in sorted(cols):
        if not c.startswith("Perf/") and c != "wall_s":
            assert [r.get(c) for r in rows["b200"]] == [r.get(c) for r in rows["upstream"]], (c, spec)


@pytest.mark.parametrize("draw", range(PARITY_DRAWS))
def test_random_models_and_extensions_log_exactly_what_upstream_logs(ref, tmp_path, draw):
    """Randomly drawn model families (MLP, GRU / LSTM, layer counts), policies (Gaussian scalar / log std,
    heteroscedastic, Beta) and extensions (RND with and without normalisation, symmetry modes)."""
    import dataclasses
    import random

    rng = random.Random(5000 + draw)
    env_name = rng.choice(["cartpole", "pendulum", "tracking12", "cartpole_po"])
    spec = dataclasses.replace(R.SPECS[env_name], num_envs=rng.choice([16, 32]), num_steps=rng.choice([4, 8]),
                               hidden=tuple(rng.choice([16, 32]) for _ in range(rng.randint(1, 2))),
                               distribution=rng.choice(["GaussianDistribution", "HeteroscedasticGaussianDistribution",
                                                        "BetaDistribution"]),
                               algorithm={**R.SPECS[env_name].algorithm,
                                          "num_learning_epochs": rng.randint(1, 3),
                                          "num_mini_batches": rng.choice([1, 2, 4])})
    recurrent = env_name == "cartpole_po" or rng.random() < 0.3
    if recurrent:
        spec = R.with_rnn(spec, rng.choice(["gru", "lstm"]), rng.choice([16, 32]), rng.choice([1, 2]),
                          critic=rng.random() < 0.7)
    elif spec.distribution == "GaussianDistribution" and rng.random() < 0.5:
        spec = dataclasses.replace(spec, model={"distribution_cfg": {"class_name": "GaussianDistribution",
                                                                     "init_std": 1.0, "std_type": "log"}},
                                   critic_model={})
    if rng.random() < 0.5:
        spec = R.with_rnd(env_name, spec)
        rnd = {**spec.algorithm["rnd_cfg"], "state_normalization": rng.random() < 0.5,
               "reward_normalization": rng.random() < 0.5}
        spec = dataclasses.replace(spec, algorithm={**spec.algorithm, "rnd_cfg": rnd})
    if not recurrent and rng.random() < 0.5:
        aug, mirror = rng.choice([(True, True), (True, False), (False, True)])
        spec = R.with_symmetry(env_name, spec, data_augmentation=aug, mirror_loss=mirror)
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        rows = {}
        for impl in ("b200", "upstream"):
            R.train(env_name, draw, str(tmp_path / impl), impl=impl, iterations=3, spec=spec)
            rows[impl] = golden.read_curve(tmp_path / impl / "metrics.csv")
    finally:
        torch.set_num_threads(threads)
    cols = {k for r in rows["upstream"] for k in r} | {k for r in rows["b200"] for k in r}
    for c in sorted(cols):
        if not c.startswith("Perf/") and c != "wall_s":
            assert [r.get(c) for r in rows["b200"]] == [r.get(c) for r in rows["upstream"]], (c, spec)


@pytest.mark.parametrize("draw", range(PARITY_DRAWS // 2))
def test_random_distillation_settings_log_exactly_what_upstream_logs(ref, tmp_path, draw):
    """Randomly drawn distillation settings (student family, loss, window length, epochs, clipping, learning rate)."""
    import random

    rng = random.Random(9000 + draw)
    student = rng.choice([None, {"class_name": "RNNModel", "rnn_type": "gru", "rnn_hidden_dim": 16},
                          {"class_name": "RNNModel", "rnn_type": "lstm", "rnn_hidden_dim": 16}])
    alg = {"loss_type": rng.choice(["mse", "huber"]), "gradient_length": rng.choice([1, 2, 3, 8]),
           "num_learning_epochs": rng.randint(1, 3), "max_grad_norm": rng.choice([None, 0.5, 1.0]),
           "learning_rate": rng.choice([3e-4, 1e-3])}
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        ckpt = R.make_teacher_checkpoint("tracking12", str(tmp_path / "t.pt"), iterations=1, num_envs=32,
                                         impl="upstream")
        rows = {}
        for impl in ("b200", "upstream"):
            R.train_distillation("tracking12", draw, str(tmp_path / impl), ckpt, impl=impl, iterations=3,
                                 algorithm=alg, student_model=student)
            rows[impl] = golden.read_curve(tmp_path / impl / "metrics.csv")
    finally:
        torch.set_num_threads(threads)
    for c in sorted({k for r in rows["upstream"] for k in r}):
        if not c.startswith("Perf/") and c != "wall_s":
            assert [r.get(c) for r in rows["b200"]] == [r.get(c) for r in rows["upstream"]], (c, alg, student)


@pytest.mark.parametrize("draw", range(8))
def test_selective_checkpoint_loading_matches_upstream(ref, tmp_path, draw):
    """Random ``load_cfg`` selections (actor, critic, optimizer, iteration, RND) of an upstream checkpoint into
    freshly built runners of both implementations: the resulting checkpoints and iteration counters are equal."""
    import dataclasses
    import random

    rng = random.Random(12000 + draw)
    spec = R.with_rnd("tracking12", dataclasses.replace(R.SPECS["tracking12"], num_envs=32, num_steps=4))
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        src, _, _ = R.build_runner("tracking12", 0, None, spec, impl="upstream")
        src.learn(2)
        src.save(str(tmp_path / "src.pt"))
        load_cfg = {k: rng.random() < 0.5 for k in ("actor", "critic", "optimizer", "iteration", "rnd")}
        saved = {}
        for impl in ("b200", "upstream"):
            dst, _, _ = R.build_runner("tracking12", 1, None, spec, impl=impl)
            dst.load(str(tmp_path / "src.pt"), load_cfg=dict(load_cfg))
            dst.save(str(tmp_path / f"{impl}.pt"))
            saved[impl] = (dst.current_learning_iteration, torch.load(tmp_path / f"{impl}.pt", weights_only=False))
    finally:
        torch.set_num_threads(threads)
    assert saved["b200"][0] == saved["upstream"][0]
    for key in saved["upstream"][1]:
        _equal_state(saved["b200"][1][key], saved["upstream"][1][key], f"{key} with {load_cfg}")


def test_distillation_checkpoint_resumes_like_upstream(ref, tmp_path):
    """A distillation checkpoint (student, teacher, optimizer) of upstream loads into both implementations, which then
    train on identically."""
    threads = torch.get_num_threads()
    torch.set_num_threads(2)
    try:
        teacher = R.make_teacher_checkpoint("tracking12", str(tmp_path / "t.pt"), iterations=1, num_envs=32,
                                            impl="upstream")
        src, _, _ = R.build_distillation_runner("tracking12", 0, None, teacher, impl="upstream", num_envs=32)
        src.learn(2)
        src.save(str(tmp_path / "distill.pt"))
        saved = {}
        for impl in ("b200", "upstream"):
            runner, _, _ = R.build_distillation_runner("tracking12", 3, None, teacher, impl=impl, num_envs=32)
            runner.load(str(tmp_path / "distill.pt"))
            runner.learn(2)
            runner.save(str(tmp_path / f"{impl}.pt"))
            saved[impl] = torch.load(tmp_path / f"{impl}.pt", weights_only=False)
    finally:
        torch.set_num_threads(threads)
    assert saved["b200"]["iter"] == saved["upstream"]["iter"]
    for key in saved["upstream"]:
        _equal_state(saved["b200"][key], saved["upstream"][key], key)


def test_golden_check_takes_the_execution_path(tmp_path):
    """``golden check --engine torch`` trains the PyTorch path (here on the CPU, where it is the only path)."""
    from tt_rsl_rl_b200.testing import golden

    out = golden.check(["cartpole"], seeds=[0], iterations=2, log_root=str(tmp_path), engine="torch",
                       mixed_precision=False)
    assert out[0]["env"] == "cartpole" and len(out[0]["final_rewards"]) == 1
    cfg = (tmp_path / "cartpole" / "seed0" / "config.json").read_text()
    assert '"engine": "torch"' in cfg
