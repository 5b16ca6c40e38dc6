"""Numerics of the RL kernels against plain PyTorch fp32 references of the same ops.

References are the upstream definitions: PPO loss (``rsl_rl/algorithms/ppo.py:241-285``, autograd gradients), GAE
(``ppo.py:166-191``), Adam + clip_grad_norm_ (torch.optim.Adam, nn.utils.clip_grad_norm_), EmpiricalNormalization.update
(``rsl_rl/modules/normalization.py:51-78``).
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def C():
    from tt_rsl_rl_b200.ops import ext

    return ext()


def _loss_reference(head, value, std_raw, log_std, hetero, actions, omean, ostd, ologp, adv, ret, vold, clip, vc, ec,
                    std_lo=1e-6, std_hi=1e6):
    A = actions.shape[1]
    head = head.clone().requires_grad_(True)
    value = value.clone().requires_grad_(True)
    std_raw = std_raw.clone().requires_grad_(True)
    if hetero:
        mean = head[:, :A]
        raw = head[:, A:]
    else:
        mean = head
        raw = std_raw
    if log_std:
        std = torch.exp(raw.clamp(math.log(std_lo), math.log(std_hi)))
    else:
        std = raw.clamp(std_lo, std_hi)
    if not hetero:
        std = std.expand_as(mean)
    dist = torch.distributions.Normal(mean, std)
    logp = dist.log_prob(actions).sum(-1)
    ent = dist.entropy().sum(-1)
    kl = torch.distributions.kl_divergence(torch.distributions.Normal(omean, ostd), dist).sum(-1).mean()
    ratio = torch.exp(logp - ologp)
    s = torch.max(-adv * ratio, -adv * torch.clamp(ratio, 1 - clip, 1 + clip)).mean()
    v = value[:, 0]
    vcl = vold + (v - vold).clamp(-clip, clip)
    vl = torch.max((v - ret).pow(2), (vcl - ret).pow(2)).mean()
    loss = s + vc * vl - ec * ent.mean()
    loss.backward()
    return dict(dhead=head.grad, dvalue=value.grad, dstd=std_raw.grad, surr=s.item(), vloss=vl.item(),
                ent=ent.mean().item(), kl=kl.item())


@pytest.mark.parametrize("hetero,log_std", [(False, False), (False, True), (True, False), (True, True)])
def test_ppo_loss_matches_autograd(hetero, log_std):
    torch.manual_seed(0)
    dev = "cuda"
    B, A, total = 1000, 29, 3000
    hc = 2 * A if hetero else A
    head = torch.randn(B, hc, device=dev) * 0.5
    if hetero:
        head[:, A:] = torch.rand(B, A, device=dev) * 0.8 + 0.3 if not log_std else torch.randn(B, A, device=dev) * 0.3
    std_raw = (torch.rand(A, device=dev) + 0.5) if not log_std else torch.randn(A, device=dev) * 0.3
    value = torch.randn(B, 1, device=dev)
    idx = torch.randperm(total, device=dev)[:B].int()
    st_actions = torch.randn(total, A, device=dev)
    st_mean = torch.randn(total, A, device=dev) * 0.5
    st_std = torch.rand(total, A, device=dev) + 0.5
    st_adv = torch.randn(total, device=dev)
    st_ret = torch.randn(total, device=dev)
    st_val = torch.randn(total, device=dev)
    # old log-probs near the new ones so that the ratio straddles the clip range
    il = idx.long()
    with torch.no_grad():
        mean = head[:, :A]
        if hetero:
            raw = head[:, A:]
            std = torch.exp(raw) if log_std else raw
        else:
            std = (torch.exp(std_raw) if log_std else std_raw).expand_as(mean)
        lp = torch.distributions.Normal(mean, std).log_prob(st_actions[il]).sum(-1)
    st_logp = torch.randn(total, device=dev) * 0.3
    st_logp[il] = lp + torch.randn(B, device=dev) * 0.3
    clip, vc, ec = 0.2, 1.0, 0.01
    ref = _loss_reference(head, value, std_raw, log_std, hetero, st_actions[il], st_mean[il], st_std[il], st_logp[il],
                          st_adv[il], st_ret[il], st_val[il], clip, vc, ec)
    blocks = C().ppo_loss_blocks(B)
    d_head = torch.zeros(B, (hc + 7) // 8 * 8, device=dev, dtype=torch.bfloat16)
    d_value = torch.zeros(B, 8, device=dev, dtype=torch.bfloat16)
    stats = torch.zeros(blocks, 5, device=dev)
    dh_col = torch.zeros(blocks, hc, device=dev)
    dv_col = torch.zeros(blocks, 1, device=dev)
    dstd = torch.zeros(blocks, A, device=dev)
    C().ppo_loss(B, A, hetero, log_std, head, hc, value, 1, None if hetero else std_raw, 1e-6, 1e6, math.log(1e-6),
                 math.log(1e6), idx, st_actions, st_mean, st_std, st_logp, st_adv, st_ret, st_val, None, clip, vc, ec,
                 True, d_head, d_head.shape[1], d_value, 8, stats, dh_col, dv_col, None if hetero else dstd, 1, False,
                 None, None, 0.0, None)
    torch.cuda.synchronize()
    scale = ref["dhead"].abs().max().item()
    torch.testing.assert_close(d_head[:, :hc].float(), ref["dhead"], atol=1e-2 * scale, rtol=1e-2)
    assert d_head[:, hc:].float().abs().max().item() == 0.0
    torch.testing.assert_close(d_value[:, 0].float(), ref["dvalue"][:, 0], atol=1e-2 * ref["dvalue"].abs().max().item(),
                               rtol=1e-2)
    torch.testing.assert_close(dh_col.sum(0), ref["dhead"].sum(0), atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(dv_col.sum(), ref["dvalue"].sum(), atol=1e-4, rtol=1e-3)
    if not hetero:
        torch.testing.assert_close(dstd.sum(0), ref["dstd"], atol=1e-5, rtol=1e-3)
    s = stats.sum(0).tolist()
    assert s[0] == pytest.approx(ref["surr"], rel=1e-4, abs=1e-5)
    assert s[1] == pytest.approx(ref["vloss"], rel=1e-4)
    assert s[2] == pytest.approx(ref["ent"], rel=1e-4)
    assert s[3] == pytest.approx(ref["kl"], rel=1e-3)


def test_gae_and_advantage_normalisation():
    torch.manual_seed(1)
    dev = "cuda"
    T, N = 24, 1000
    rewards = torch.randn(T, N, device=dev)
    dones = (torch.rand(T, N, device=dev) < 0.05).float()
    values = torch.randn(T, N, device=dev)
    last = torch.randn(N, device=dev)
    gamma, lam = 0.99, 0.95
    # reference (upstream loop)
    ret_ref = torch.zeros(T, N, device=dev)
    adv = torch.zeros(N, device=dev)
    for t in reversed(range(T)):
        nv = last if t == T - 1 else values[t + 1]
        nd = 1.0 - dones[t]
        delta = rewards[t] + nd * gamma * nv - values[t]
        adv = delta + nd * gamma * lam * adv
        ret_ref[t] = adv + values[t]
    adv_ref = ret_ref - values
    adv_ref = (adv_ref - adv_ref.mean()) / (adv_ref.std() + 1e-8)
    ret = torch.zeros(T * N, device=dev)
    advs = torch.zeros(T * N, device=dev)
    part = torch.zeros(2 * C().gae_blocks(N), dtype=torch.float64, device=dev)
    C().gae(rewards.view(-1), dones.view(-1), values.view(-1), last, ret, advs, T, N, gamma, lam, part)
    C().adv_normalize(advs, part, C().gae_blocks(N))
    torch.cuda.synchronize()
    torch.testing.assert_close(ret.view(T, N), ret_ref, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(advs.view(T, N), adv_ref, atol=1e-5, rtol=1e-4)


def test_gather_feistel_permutation_and_normalisation():
    torch.manual_seed(2)
    dev = "cuda"
    total, M = 24 * 1001, 4
    hb = C().feistel_half_bits(total)
    obs_a = torch.randn(total, 96, device=dev)
    obs_c = torch.randn(total, 99, device=dev)
    mean_a, std_a = torch.randn(96, device=dev), torch.rand(96, device=dev) + 0.5
    key = torch.tensor([12345], dtype=torch.int32, device=dev)
    seen = []
    for i in range(M):
        start = i * total // M
        B = (i + 1) * total // M - start
        idx = torch.zeros(B, dtype=torch.int32, device=dev)
        xa = torch.zeros(B, 96, device=dev, dtype=torch.bfloat16)
        xc = torch.zeros(B, 104, device=dev, dtype=torch.bfloat16)
        C().gather_minibatch(B, start, total, key, hb, None, idx, [obs_a, obs_c], [mean_a, None], [std_a, None], 1e-2,
                             [xa, xc], [96, 104], None, 1, [B, B], [None, None], [None, None])
        torch.cuda.synchronize()
        il = idx.long()
        seen.append(il)
        ref_a = (obs_a[il] - mean_a) / (std_a + 1e-2)
        torch.testing.assert_close(xa.float(), ref_a, atol=2e-2, rtol=1e-2)
        torch.testing.assert_close(xc[:, :99].float(), obs_c[il], atol=2e-2, rtol=1e-2)
        # host implementation of the same permutation agrees
        for j in (0, B // 2, B - 1):
            assert int(il[j]) == C().feistel_permute(start + j, total, hb, 12345)
    allidx = torch.cat(seen)
    assert torch.equal(torch.sort(allidx).values, torch.arange(total, device=dev))


def test_adam_with_two_clip_groups_matches_torch():
    torch.manual_seed(3)
    dev = "cuda"
    shapes = [(512, 96), (512,), (29, 128), (29,), (256, 99), (1,)]
    groups = [0, 0, 0, 0, 1, 1]
    params = [torch.randn(*s, device=dev) * 0.1 for s in shapes]
    offsets, off = [], 0
    for p in params:
        offsets.append(off)
        off += p.numel()
    n = off
    flat = torch.cat([p.reshape(-1) for p in params])
    ref_params = [torch.nn.Parameter(p.clone()) for p in params]
    opt = torch.optim.Adam(ref_params, lr=1e-3)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    n_ex = (n + 4 + 3) // 4 * 4
    send = torch.zeros(n_ex, device=dev)
    grads = torch.zeros(n_ex, device=dev)
    shadows = [torch.zeros(s[0], (s[1] + 7) // 8 * 8, device=dev, dtype=torch.bfloat16) if len(s) == 2 else None
               for s in shapes]
    tens, chunks, nch = C().make_adam_plan(
        offsets + [n], [p.numel() for p in params] + [4], groups + [-1],
        [s[0] if len(s) == 2 else 1 for s in shapes] + [1], [s[1] if len(s) == 2 else s[0] for s in shapes] + [4],
        shadows + [None], [sh.shape[1] if sh is not None else 0 for sh in shadows] + [0], flat)
    grid = C().adam_grid(torch.cuda.current_device())
    lr = torch.tensor([1e-3, 1e-3], device=dev)
    step = torch.zeros(2, dtype=torch.int64, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    norm_partial = torch.zeros(grid * 4, device=dev)
    barrier = torch.zeros(4, dtype=torch.int32, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    for it in range(3):
        gs = [torch.randn(*s, device=dev) * (3.0 if it == 0 else 0.01) for s in shapes]
        send[:n] = torch.cat([g.reshape(-1) for g in gs])
        send[n + 3] = 0.005  # KL inside the band: learning rate unchanged
        C().adam_step(flat, send, send, grads, m, v, tens, chunks, nch, [1.0, 1.0], [0.9, 0.9], [0.999, 0.999],
                      [1e-8, 1e-8], [0, 0], lr, None, step, True, grads[n + 3 : n + 4], 0.01, 1e-5, 1e-2, 1, 0, None,
                      None, epoch, 10**9, norm_partial, barrier, status, None, grid, [0, offsets[4], offsets[4], n],
                      n_ex, None, -1)
        for p, g in zip(ref_params, gs):
            p.grad = g.clone()
        torch.nn.utils.clip_grad_norm_([ref_params[i] for i in range(6) if groups[i] == 0], 1.0)
        torch.nn.utils.clip_grad_norm_([ref_params[i] for i in range(6) if groups[i] == 1], 1.0)
        opt.step()
    torch.cuda.synchronize()
    assert status[0].item() == 0
    ref_flat = torch.cat([p.detach().reshape(-1) for p in ref_params])
    torch.testing.assert_close(flat, ref_flat, atol=2e-6, rtol=1e-5)
    assert int(step[0]) == 3 and int(epoch[0]) == 3
    for i, (sh, s) in enumerate(zip(shadows, shapes)):
        if sh is not None:
            o = offsets[i]
            w = flat[o : o + params[i].numel()].view(*s)
            torch.testing.assert_close(sh[:, : s[1]].float(), w.bfloat16().float())


def test_adaptive_learning_rate_rule():
    dev = "cuda"
    n = 64
    flat = torch.zeros(n, device=dev)
    tens, chunks, nch = C().make_adam_plan([0, n], [n, 4], [0, -1], [1, 1], [n, 4], [None, None], [0, 0], flat)
    grid = C().adam_grid(torch.cuda.current_device())
    lr = torch.tensor([1e-3, 1e-3], device=dev)
    args = dict(step=torch.zeros(2, dtype=torch.int64, device=dev), epoch=torch.zeros(1, dtype=torch.int32, device=dev),
                norm_partial=torch.zeros(grid * 4, device=dev), barrier=torch.zeros(4, dtype=torch.int32, device=dev))
    send = torch.zeros(n + 4, device=dev)
    grads = torch.zeros(n + 4, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    expect = 1e-3
    for kl in (0.05, 0.05, 0.001, 0.0, 0.01):
        send[n + 3] = kl
        C().adam_step(flat, send, send, grads, m, v, tens, chunks, nch, [1.0], [0.9], [0.999], [1e-8], [0], lr, None,
                      args["step"], True, grads[n + 3 : n + 4], 0.01, 1e-5, 1e-2, 1, 0, None, None, args["epoch"],
                      10**9, args["norm_partial"], args["barrier"], None, None, grid, [0, n], n + 4, None, -1)
        if kl > 0.02:
            expect = max(1e-5, expect / 1.5)
        elif 0.0 < kl < 0.005:
            expect = min(1e-2, expect * 1.5)
        torch.cuda.synchronize()
        assert lr[0].item() == pytest.approx(expect, rel=1e-5)


def test_normalizer_update_matches_module():
    from tt_rsl_rl_b200.modules import EmpiricalNormalization

    torch.manual_seed(4)
    dev = "cuda"
    D, rows = 99, 20000
    ref = EmpiricalNormalization(D).to(dev)
    mine = EmpiricalNormalization(D).to(dev)
    for it in range(3):
        x = torch.randn(rows, D, device=dev) * (it + 1) + it
        ref.update(x)
        chunks = C().colstats_chunks(rows)
        part = torch.zeros(2 * chunks * D, dtype=torch.float64, device=dev)
        C().colstats(x, rows, D, D, part)
        C().norm_update(part, chunks, rows, D, mine._mean.view(-1), mine._var.view(-1), mine._std.view(-1), mine.count,
                        -1, None, False)
    torch.cuda.synchronize()
    assert int(mine.count) == int(ref.count)
    torch.testing.assert_close(mine._mean, ref._mean, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(mine._var, ref._var, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(mine._std, ref._std, atol=1e-4, rtol=1e-4)


def test_gaussian_sample_statistics_and_logprob():
    torch.manual_seed(5)
    dev = "cuda"
    N, A = 200000, 29
    head = torch.randn(N, A, device=dev)
    std = torch.rand(A, device=dev) + 0.5
    counter = torch.zeros(1, dtype=torch.int64, device=dev)
    ticket = torch.zeros(1, dtype=torch.int32, device=dev)
    act = torch.zeros(N, A, device=dev)
    om = torch.zeros(N, A, device=dev)
    osd = torch.zeros(N, A, device=dev)
    lp = torch.zeros(N, device=dev)
    C().gaussian_sample(head, A, N, A, False, False, std, 1e-6, 1e6, math.log(1e-6), math.log(1e6), 7, counter, ticket,
                        act, om, osd, lp, None)
    torch.cuda.synchronize()
    z = (act - head) / std
    assert abs(z.mean().item()) < 5e-3
    assert abs(z.std().item() - 1.0) < 5e-3
    ref_lp = torch.distributions.Normal(head, std).log_prob(act).sum(-1)
    torch.testing.assert_close(lp, ref_lp, atol=1e-3, rtol=1e-4)
    torch.testing.assert_close(om, head)
    assert int(counter.item()) == 1
    # a second call draws fresh noise
    act2 = torch.zeros_like(act)
    C().gaussian_sample(head, A, N, A, False, False, std, 1e-6, 1e6, math.log(1e-6), math.log(1e6), 7, counter, ticket,
                        act2, om, osd, lp, None)
    torch.cuda.synchronize()
    assert not torch.equal(act, act2)
