"""Kernels of the symmetry and RND extensions against plain PyTorch fp32 references: mirrored minibatch gather,
the PPO loss with augmented copies and the mirror loss, and the RND intrinsic reward."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def C():
    from tt_rsl_rl_b200.ops import ext

    return ext()


def _signed_perms(K, D, gen):
    """Copy 0 identity; copies 1.. random involutive-free signed permutations."""
    perm = [torch.arange(D)]
    sign = [torch.ones(D)]
    for _ in range(1, K):
        perm.append(torch.randperm(D, generator=gen))
        sign.append(torch.where(torch.rand(D, generator=gen) < 0.5, -1.0, 1.0))
    return torch.stack(perm).int().cuda(), torch.stack(sign).cuda()


def _apply(x, perm, sign):
    return x[:, perm.long()] * sign


@pytest.mark.parametrize("K", [2, 3])
def test_gather_writes_mirrored_copies(K):
    gen = torch.Generator().manual_seed(0)
    dev = "cuda"
    total, B = 4000, 1000
    obs_a = torch.randn(total, 40, device=dev)
    obs_c = torch.randn(total, 43, device=dev)
    mean_a, std_a = torch.randn(40, device=dev), torch.rand(40, device=dev) + 0.5
    perm_a, sign_a = _signed_perms(K, 40, gen)
    perm_c, sign_c = _signed_perms(K, 43, gen)
    idx_in = torch.randperm(total, device=dev)[:B].int()
    idx = torch.zeros(B, dtype=torch.int32, device=dev)
    xa = torch.zeros(K * B, 40, device=dev, dtype=torch.bfloat16)
    xc = torch.zeros(K * B, 48, device=dev, dtype=torch.bfloat16)
    xr = torch.zeros(B, 48, device=dev, dtype=torch.bfloat16)
    C().gather_minibatch(B, 0, total, None, C().feistel_half_bits(total), idx_in, idx, [obs_a, obs_c, obs_c],
                         [mean_a, None, None], [std_a, None, None], 1e-2, [xa, xc, xr], [40, 48, 48], None, K,
                         [K * B, K * B, B], [perm_a, perm_c, None], [sign_a, sign_c, None])
    torch.cuda.synchronize()
    il = idx_in.long()
    assert torch.equal(idx, idx_in)
    for k in range(K):
        ref_a = (_apply(obs_a[il], perm_a[k], sign_a[k]) - mean_a) / (std_a + 1e-2)
        torch.testing.assert_close(xa[k * B : (k + 1) * B].float(), ref_a, atol=3e-2, rtol=1e-2)
        ref_c = _apply(obs_c[il], perm_c[k], sign_c[k])
        torch.testing.assert_close(xc[k * B : (k + 1) * B, :43].float(), ref_c, atol=3e-2, rtol=1e-2)
    torch.testing.assert_close(xr[:, :43].float(), obs_c[il], atol=3e-2, rtol=1e-2)


@pytest.mark.parametrize("aug,K,coef", [(True, 2, 1.0), (False, 2, 0.5), (True, 3, 0.0)])
def test_ppo_loss_with_symmetry_matches_autograd(aug, K, coef):
    gen = torch.Generator().manual_seed(1)
    torch.manual_seed(1)
    dev = "cuda"
    n0, A, total = 700, 12, 3000
    rows = K * n0
    rows_c = rows if aug else n0
    perm, sign = _signed_perms(K, A, gen)
    head = (torch.randn(rows, A, device=dev) * 0.5).requires_grad_(True)
    std_raw = (torch.rand(A, device=dev) + 0.5).requires_grad_(True)
    value = torch.randn(rows_c, 1, device=dev).requires_grad_(True)
    idx = torch.randperm(total, device=dev)[:n0].int()
    il = idx.long()
    st_actions = torch.randn(total, A, device=dev)
    st_mean = torch.randn(total, A, device=dev) * 0.5
    st_std = torch.rand(total, A, device=dev) + 0.5
    st_adv, st_ret, st_val = (torch.randn(total, device=dev) for _ in range(3))
    clip, vc, ec = 0.2, 1.0, 0.01
    # upstream semantics: augment_batch + compute_loss
    acts = torch.cat([_apply(st_actions[il], perm[k], sign[k]) for k in range(K)])
    std = std_raw.expand(rows, A)
    with torch.no_grad():  # old log-probs near the new ones so that the ratio straddles the clip range
        lp0 = torch.distributions.Normal(head[:n0], std[:n0]).log_prob(acts[:n0]).sum(-1)
    st_logp = torch.randn(total, device=dev) * 0.3
    st_logp[il] = lp0 + torch.randn(n0, device=dev) * 0.3
    dist = torch.distributions.Normal(head, std)
    logp = dist.log_prob(acts).sum(-1)
    ent = dist.entropy().sum(-1)[:n0]
    rep = K if aug else 1
    old_lp = st_logp[il].repeat(rep)
    adv = st_adv[il].repeat(rep)
    ret = st_ret[il].repeat(rep)
    vold = st_val[il].repeat(rep)
    ratio = torch.exp(logp[: rep * n0] - old_lp)
    surr = torch.max(-adv * ratio, -adv * torch.clamp(ratio, 1 - clip, 1 + clip)).mean()
    v = value[:, 0]
    vcl = vold + (v - vold).clamp(-clip, clip)
    vl = torch.max((v - ret).pow(2), (vcl - ret).pow(2)).mean()
    loss = surr + vc * vl - ec * ent.mean()
    mirrored = torch.cat([_apply(head[:n0].detach(), perm[k], sign[k]) for k in range(1, K)])
    sym = torch.nn.functional.mse_loss(head[n0:], mirrored)
    loss = loss + coef * sym
    loss.backward()
    kl = torch.distributions.kl_divergence(torch.distributions.Normal(st_mean[il], st_std[il]),
                                           torch.distributions.Normal(head[:n0].detach(), std[:n0].detach()))
    kl = kl.sum(-1).mean()

    blocks = C().ppo_loss_blocks(rows)
    d_head = torch.zeros(rows, 16, device=dev, dtype=torch.bfloat16)
    d_value = torch.zeros(rows_c, 8, device=dev, dtype=torch.bfloat16)
    stats = torch.zeros(blocks, 5, device=dev)
    dh_col = torch.zeros(blocks, A, device=dev)
    dv_col = torch.zeros(blocks, 1, device=dev)
    dstd = torch.zeros(blocks, A, device=dev)
    C().ppo_loss(n0, A, False, False, head.detach(), A, value.detach(), 1, std_raw.detach(), 1e-6, 1e6,
                 math.log(1e-6), math.log(1e6), idx, st_actions, st_mean, st_std, st_logp, st_adv, st_ret, st_val, None,
                 clip, vc, ec, True, d_head, 16, d_value, 8, stats, dh_col, dv_col, dstd, K, aug, perm, sign, coef,
                 None)
    torch.cuda.synchronize()
    scale = head.grad.abs().max().item()
    torch.testing.assert_close(d_head[:, :A].float(), head.grad, atol=1e-2 * scale, rtol=1e-2)
    torch.testing.assert_close(d_value[:, 0].float(), value.grad[:, 0], atol=1e-2 * value.grad.abs().max().item(),
                               rtol=1e-2)
    torch.testing.assert_close(dh_col.sum(0), head.grad.sum(0), atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(dstd.sum(0), std_raw.grad, atol=1e-5, rtol=1e-3)
    s = stats.sum(0).tolist()
    assert s[0] == pytest.approx(surr.item(), rel=1e-4, abs=1e-5)
    assert s[1] == pytest.approx(vl.item(), rel=1e-4)
    assert s[2] == pytest.approx(ent.mean().item(), rel=1e-4)
    assert s[3] == pytest.approx(kl.item(), rel=1e-3)
    assert s[4] == pytest.approx(sym.item(), rel=1e-4)


def test_rnd_intrinsic_reward():
    torch.manual_seed(2)
    t = torch.randn(5000, 16, device="cuda")
    p = torch.randn(5000, 16, device="cuda")
    w = torch.tensor([0.37, 9.0], device="cuda")
    out = torch.zeros(5000, device="cuda")
    C().rnd_intrinsic(t, 16, p, 16, 5000, 16, w[0:1], out, None, 0.0)
    torch.testing.assert_close(out, 0.37 * torch.linalg.norm(t - p, dim=1), rtol=1e-5, atol=1e-6)
    # normalised form: raw distance + discounted sum, then weight / std
    disc = torch.full((5000,), 0.5, device="cuda")
    C().rnd_intrinsic(t, 16, p, 16, 5000, 16, w[0:1], out, disc, 0.9)
    raw = torch.linalg.norm(t - p, dim=1)
    torch.testing.assert_close(out, raw, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(disc, 0.45 + raw, rtol=1e-5, atol=1e-6)
    std = torch.tensor([2.5], device="cuda")
    C().rnd_reward_scale(out, 5000, w[0:1], std)
    torch.testing.assert_close(out, 0.37 * raw / 2.5, rtol=1e-5, atol=1e-6)
