"""Numerics of the tcgen05 GEMM against a plain PyTorch fp32 reference of the same op (bf16-rounded operands)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().t()


def _bf16(shape, scale=1.0, gen=None):
    return (torch.randn(*shape, generator=gen, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (300, 512, 96), (1000, 29, 128), (4099, 256, 512), (257, 1, 256),
                                   (513, 128, 99), (64, 32, 200)])
def test_forward_f32_bias(M, N, K):
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(0)
    kp = G.pad8(K)
    x = torch.zeros(M, kp, device="cuda", dtype=torch.bfloat16)
    x[:, :K] = _bf16((M, K))
    w = torch.zeros(N, kp, device="cuda", dtype=torch.bfloat16)
    w[:, :K] = _bf16((N, K), 0.1)
    bias = torch.randn(N, device="cuda")
    out = torch.full((M, N), float("nan"), device="cuda")
    G.gemm(x, kp, False, w, kp, False, M, N, K, G.EPI_F32, out, N, bias=bias)
    torch.cuda.synchronize()
    ref = _ref(x[:, :K], w[:, :K]) + bias
    torch.testing.assert_close(out, ref, atol=2e-3 * (K ** 0.5), rtol=1e-3)
    # same bf16 operands on both sides: only the fp32 accumulation order differs
    from tt_rsl_rl_b200.testing import assert_parity

    assert_parity(out, ref, "fp32_elementwise", f"gemm fp32 epilogue {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(1000, 29, 128), (300, 58, 96), (77, 1, 64)])
def test_forward_f32_padded_output_columns(M, N, K):
    """out_cols: a row pitch rounded up to 32-column chunks takes whole chunks (zeros past N), nothing past out_cols."""
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(2)
    kp = G.pad8(K)
    x = torch.zeros(M, kp, device="cuda", dtype=torch.bfloat16)
    x[:, :K] = _bf16((M, K))
    w = torch.zeros(N, kp, device="cuda", dtype=torch.bfloat16)
    w[:, :K] = _bf16((N, K), 0.1)
    bias = torch.randn(N, device="cuda")
    pitch = (N + 31) // 32 * 32
    out = torch.full((M, pitch + 8), float("nan"), device="cuda")  # 8 columns beyond the writable ones
    G.gemm(x, kp, False, w, kp, False, M, N, K, G.EPI_F32, out, pitch + 8, bias=bias, out_cols=pitch)
    torch.cuda.synchronize()
    ref = _ref(x[:, :K], w[:, :K]) + bias
    torch.testing.assert_close(out[:, :N], ref, atol=2e-3 * (K ** 0.5), rtol=1e-3)
    pad = out[:, N:pitch]
    assert ((pad == 0) | pad.isnan()).all()  # zeros where a whole chunk was stored, untouched otherwise
    assert out[:, pitch:].isnan().all()


@pytest.mark.parametrize("M,N,K", [(300, 512, 96), (1000, 256, 512), (129, 128, 256), (77, 40, 64)])
def test_forward_bias_elu_bf16(M, N, K):
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(1)
    x = _bf16((M, K))
    w = _bf16((N, K), 0.1)
    bias = torch.randn(N, device="cuda") * 0.1
    np_ = G.pad8(N)
    out = torch.zeros(M, np_, device="cuda", dtype=torch.bfloat16)
    G.gemm(x, K, False, w, K, False, M, N, K, G.EPI_BIAS_ELU_BF16, out, np_, bias=bias)
    torch.cuda.synchronize()
    ref = torch.nn.functional.elu(_ref(x, w) + bias)
    torch.testing.assert_close(out[:, :N].float(), ref, atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("M,Nin,Kout", [(777, 512, 256), (4096, 128, 29), (300, 256, 128), (65, 96, 512)])
def test_dgrad_elu_colsum(M, Nin, Kout):
    """dZ_in = (dZ_out @ W) * elu'(H_in) with W [Kout, Nin] read MN-major; column sums of dZ_in per 128-row tile."""
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(2)
    kp = G.pad8(Kout)
    dz = torch.zeros(M, kp, device="cuda", dtype=torch.bfloat16)
    dz[:, :Kout] = _bf16((M, Kout))
    w = _bf16((Kout, Nin), 0.1)
    h = torch.nn.functional.elu(torch.randn(M, Nin, device="cuda")).to(torch.bfloat16)
    out = torch.zeros(M, Nin, device="cuda", dtype=torch.bfloat16)
    colsum = torch.full((G.colsum_rows(), Nin), float("nan"), device="cuda")  # every row is written
    G.gemm(dz, kp, False, w, Nin, True, M, Nin, Kout, G.EPI_DGRAD_ELU, out, Nin, aux=h, ld_aux=Nin, colsum=colsum)
    torch.cuda.synchronize()
    hf = h.float()
    grad = torch.where(hf > 0, torch.ones_like(hf), hf + 1)
    ref = (dz[:, :Kout].float() @ w.float()) * grad
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(colsum.sum(0), ref.sum(0), atol=1e-2 * M ** 0.5, rtol=1e-3)


@pytest.mark.parametrize("M,Nin,Kout", [(333, 40, 64), (130, 72, 29), (200, 36, 64)])
def test_dgrad_elu_padded_pitches(M, Nin, Kout):
    """Output and activation buffers with different padded row pitches: padding columns are left untouched."""
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(5)
    kp = G.pad8(Kout)
    dz = torch.zeros(M, kp, device="cuda", dtype=torch.bfloat16)
    dz[:, :Kout] = _bf16((M, Kout))
    w = _bf16((Kout, G.pad8(Nin) + 8), 0.1)
    h = torch.zeros(M, G.pad8(Nin) + 8, device="cuda", dtype=torch.bfloat16)
    h[:, :Nin] = torch.nn.functional.elu(torch.randn(M, Nin, device="cuda")).to(torch.bfloat16)
    out = torch.full((M, G.pad8(Nin) + 16), 7.0, device="cuda", dtype=torch.bfloat16)
    colsum = torch.full((G.colsum_rows(), Nin), float("nan"), device="cuda")  # every row is written
    G.gemm(dz, kp, False, w, w.shape[1], True, M, Nin, Kout, G.EPI_DGRAD_ELU, out, out.shape[1], aux=h,
           ld_aux=h.shape[1], colsum=colsum)
    torch.cuda.synchronize()
    hf = h[:, :Nin].float()
    grad = torch.where(hf > 0, torch.ones_like(hf), hf + 1)
    ref = (dz[:, :Kout].float() @ w[:, :Nin].float()) * grad
    torch.testing.assert_close(out[:, :Nin].float(), ref, atol=3e-2, rtol=2e-2)
    assert (out[:, Nin : G.pad8(Nin)].float() == 0.0).all()
    assert (out[:, G.pad8(Nin) :].float() == 7.0).all()
    torch.testing.assert_close(colsum.sum(0), ref.sum(0), atol=1e-2 * M ** 0.5, rtol=1e-3)


def test_forward_bias_elu_leaves_padding():
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(6)
    M, N, K = 200, 36, 64
    x = _bf16((M, K))
    w = _bf16((N, K), 0.1)
    bias = torch.randn(N, device="cuda") * 0.1
    out = torch.full((M, 48), 5.0, device="cuda", dtype=torch.bfloat16)
    G.gemm(x, K, False, w, K, False, M, N, K, G.EPI_BIAS_ELU_BF16, out, 48, bias=bias)
    torch.cuda.synchronize()
    ref = torch.nn.functional.elu(_ref(x, w) + bias)
    torch.testing.assert_close(out[:, :N].float(), ref, atol=3e-2, rtol=2e-2)
    # bf16 outputs are stored in 16-byte column groups: [N, pad8(N)) receives zeros, columns past it are untouched
    assert (out[:, N : G.pad8(N)].float() == 0.0).all()
    assert (out[:, G.pad8(N) :].float() == 5.0).all()


@pytest.mark.parametrize("rows,out_f,in_f,splits", [(4096, 256, 512, 4), (3000, 29, 128, 3), (8192, 512, 96, 8),
                                                    (1000, 1, 256, 2)])
def test_wgrad_split_partials(rows, out_f, in_f, splits):
    """dW[out, in] = dZ^T H with both operands read MN-major from row-major [rows, features] buffers."""
    from tt_rsl_rl_b200.ops import gemm as G

    torch.manual_seed(3)
    op = G.pad8(out_f)
    ip = G.pad8(in_f)
    dz = torch.zeros(rows, op, device="cuda", dtype=torch.bfloat16)
    dz[:, :out_f] = _bf16((rows, out_f))
    h = torch.zeros(rows, ip, device="cuda", dtype=torch.bfloat16)
    h[:, :in_f] = _bf16((rows, in_f))
    part = torch.full((splits, out_f, in_f), float("nan"), device="cuda")
    G.gemm(dz, op, True, h, ip, True, out_f, in_f, rows, G.EPI_PARTIAL_F32, part, in_f, splits=splits,
           split_stride=out_f * in_f)
    torch.cuda.synchronize()
    ref = dz[:, :out_f].float().t() @ h[:, :in_f].float()
    torch.testing.assert_close(part.sum(0), ref, atol=2e-3 * rows ** 0.5, rtol=1e-3)
