"""GRU / LSTM cell kernels against fp32 autograd of the torch.nn.GRU / torch.nn.LSTM step equations."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def C():
    from tt_rsl_rl_b200.ops import ext

    return ext()


def _step_ref(lstm, gi, gh, h, c):
    H = h.shape[1]
    if not lstm:
        r = torch.sigmoid(gi[:, :H] + gh[:, :H])
        z = torch.sigmoid(gi[:, H : 2 * H] + gh[:, H : 2 * H])
        n = torch.tanh(gi[:, 2 * H :] + r * gh[:, 2 * H :])
        return (1 - z) * n + z * h, None
    i = torch.sigmoid(gi[:, :H] + gh[:, :H])
    f = torch.sigmoid(gi[:, H : 2 * H] + gh[:, H : 2 * H])
    g = torch.tanh(gi[:, 2 * H : 3 * H] + gh[:, 2 * H : 3 * H])
    o = torch.sigmoid(gi[:, 3 * H :] + gh[:, 3 * H :])
    c2 = f * c + i * g
    return o * torch.tanh(c2), c2


@pytest.mark.parametrize("lstm", [False, True])
def test_cell_forward_and_masks(lstm):
    torch.manual_seed(0)
    rows, H = 1000, 256
    G, S = (4, 5) if lstm else (3, 4)
    gi = torch.randn(rows, G * H, device="cuda")
    gh = torch.randn(rows, G * H, device="cuda")
    h = torch.randn(rows, H, device="cuda")
    c = torch.randn(rows, H, device="cuda") if lstm else None
    done = (torch.rand(rows, device="cuda") < 0.3).float()
    h_out = torch.zeros(rows, H, device="cuda")
    h_bf = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    c_out = torch.zeros(rows, H, device="cuda") if lstm else None
    nh = torch.zeros(rows, H, device="cuda")
    nh_bf = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
    nc = torch.zeros(rows, H, device="cuda") if lstm else None
    save = torch.zeros(rows, S * H, device="cuda")
    C().rnn_cell_fwd(rows, H, lstm, gi, G * H, gh, G * H, h, H, c, H, h_out, H, h_bf, H, c_out, H, done, nh, H, nh_bf,
                     H, nc, H, save, S * H)
    torch.cuda.synchronize()
    ref_h, ref_c = _step_ref(lstm, gi, gh, h, c)
    torch.testing.assert_close(h_out, ref_h, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(h_bf.float(), ref_h, rtol=1e-2, atol=1e-2)
    keep = (1 - done)[:, None]
    torch.testing.assert_close(nh, ref_h * keep, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(nh_bf.float(), ref_h * keep, rtol=1e-2, atol=1e-2)
    if lstm:
        torch.testing.assert_close(c_out, ref_c, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(nc, ref_c * keep, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(save[:, 4 * H :], torch.tanh(ref_c), rtol=1e-5, atol=1e-5)
    # in-place rollout form: state updated where it is read
    st = h.clone()
    stc = c.clone() if lstm else None
    C().rnn_cell_fwd(rows, H, lstm, gi, G * H, gh, G * H, st, H, stc, H, st, H, None, 0, stc, H, None, None, 0, None, 0,
                     None, 0, None, 0)
    torch.testing.assert_close(st, ref_h, rtol=1e-5, atol=1e-5)
    # state masking
    C().rnn_mask(rows, H, st, H, stc, H, done, st, H, h_bf, H, stc, H)
    torch.testing.assert_close(st, ref_h * keep, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("lstm", [False, True])
@pytest.mark.parametrize("H", [256, 480, 1024])
def test_cell_backward_matches_autograd(lstm, H):
    torch.manual_seed(1)
    rows = 700
    G, S = (4, 5) if lstm else (3, 4)
    gi = torch.randn(rows, G * H, device="cuda", requires_grad=True)
    gh = torch.randn(rows, G * H, device="cuda", requires_grad=True)
    h = torch.randn(rows, H, device="cuda", requires_grad=True)
    c = torch.randn(rows, H, device="cuda", requires_grad=True) if lstm else None
    done = (torch.rand(rows, device="cuda") < 0.3).float()
    keep = (1 - done)[:, None]
    dh_head = torch.randn(rows, H, device="cuda")
    rec_a = torch.randn(rows, H, device="cuda")
    rec_b = torch.randn(rows, H, device="cuda")
    dc_rec = torch.randn(rows, H, device="cuda") if lstm else None
    h2, c2 = _step_ref(lstm, gi, gh, h, c)
    # h' feeds the loss directly (dh_head) and, masked, the next step (rec_a + rec_b; dc_rec for the cell state)
    loss = (h2 * dh_head).sum() + ((h2 * keep) * (rec_a + rec_b)).sum()
    if lstm:
        loss = loss + ((c2 * keep) * dc_rec).sum()
    loss.backward()
    save = torch.zeros(rows, S * H, device="cuda")
    with torch.no_grad():
        C().rnn_cell_fwd(rows, H, lstm, gi, G * H, gh, G * H, h, H, c, H, None, 0, None, 0,
                         torch.zeros(rows, H, device="cuda") if lstm else None, H, None, None, 0, None, 0, None, 0,
                         save, S * H)
    blocks = C().rnn_bwd_blocks(rows)
    dgi = torch.zeros(rows, G * H, device="cuda", dtype=torch.bfloat16)
    dgh = None if lstm else torch.zeros(rows, G * H, device="cuda", dtype=torch.bfloat16)
    dh_direct = None if lstm else torch.zeros(rows, H, device="cuda")
    dc_prev = torch.zeros(rows, H, device="cuda") if lstm else None
    cs_gi = torch.zeros(blocks, G * H, device="cuda")
    cs_gh = None if lstm else torch.zeros(blocks, G * H, device="cuda")
    C().rnn_cell_bwd(rows, H, lstm, save, S * H, None if lstm else h.detach(), H, c.detach() if lstm else None, H,
                     dh_head, H, rec_a, rec_b, H, dc_rec, H, done, dgi, G * H, dgh, G * H, dh_direct, H, dc_prev, H,
                     cs_gi, cs_gh, False)
    torch.cuda.synchronize()
    tol = dict(rtol=2e-2, atol=2e-2 * gi.grad.abs().max().item() / 8)
    torch.testing.assert_close(dgi.float(), gi.grad, **tol)
    torch.testing.assert_close(cs_gi.sum(0), gi.grad.sum(0), rtol=1e-4, atol=1e-3)
    if lstm:
        torch.testing.assert_close(gh.grad, gi.grad)  # hidden-side gradients equal the input-side ones
        torch.testing.assert_close(dc_prev, c.grad, rtol=1e-4, atol=1e-4)
    else:
        torch.testing.assert_close(dgh.float(), gh.grad, **tol)
        torch.testing.assert_close(cs_gh.sum(0), gh.grad.sum(0), rtol=1e-4, atol=1e-3)
        torch.testing.assert_close(dh_direct, h.grad, rtol=1e-4, atol=1e-4)  # dL/dh not through W_hh
    # accumulate mode adds a second sweep step's sums onto the same rows
    before = [t.clone() for t in (cs_gi, cs_gh) if t is not None]
    C().rnn_cell_bwd(rows, H, lstm, save, S * H, None if lstm else h.detach(), H, c.detach() if lstm else None, H,
                     dh_head, H, rec_a, rec_b, H, dc_rec, H, done, dgi, G * H, dgh, G * H, dh_direct, H, dc_prev, H,
                     cs_gi, cs_gh, True)
    for t, b in zip([t for t in (cs_gi, cs_gh) if t is not None], before):
        torch.testing.assert_close(t, 2 * b, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("lstm", [False, True])
@pytest.mark.parametrize("H", [128, 256])
def test_fused_step_matches_gemm_plus_cell(lstm, H):
    """One launch (hidden GEMM with the cell in its epilogue) equals the tcgen05 GEMM followed by the cell kernel, on
    env-major strided views where the next step's state goes to the next slot of the input state's buffer."""
    from tt_rsl_rl_b200.ops import gemm as Gm

    torch.manual_seed(1)
    rows, T, t = 1000, 3, 1
    G, S = (4, 5) if lstm else (3, 4)
    GH = G * H
    f32 = dict(device="cuda", dtype=torch.float32)
    hbf_buf = (torch.randn(rows, T, H, **f32) * 0.5).bfloat16()  # input state at slot t, next state to slot t + 1
    h_buf = torch.randn(rows, T, H, **f32) * 0.5
    c_buf = torch.randn(rows, T, H, **f32) if lstm else None
    gi_buf = torch.randn(rows, T, GH, **f32)
    w = (torch.randn(GH, H, **f32) / H**0.5).bfloat16()
    b = torch.randn(GH, **f32) * 0.1
    done = (torch.rand(rows, device="cuda") < 0.2).float()
    status = torch.zeros(4, dtype=torch.int32, device="cuda")

    def view(buf, slot):
        return buf.view(-1)[slot * buf.shape[2] :]

    outs = {}
    for fused in (True, False):
        hb = hbf_buf.clone()
        hout_bf = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
        nh = torch.zeros(rows, T, H, **f32)
        nc = torch.zeros(rows, T, H, **f32) if lstm else None
        save = torch.zeros(rows, S * H, **f32)
        c_in = (view(c_buf, t), T * H) if lstm else (None, 0)
        c_next = (view(nc, t + 1), T * H) if lstm else (None, 0)
        if fused:
            C().rnn_step_fused(rows, H, lstm, view(hb, t), T * H, w, H, b, view(gi_buf, t), T * GH, view(h_buf, t),
                               T * H, *c_in, None, 0, hout_bf, H, None, 0, done, view(nh, t + 1), T * H,
                               view(hb, t + 1), T * H, *c_next, save, S * H, status)
        else:
            gh = torch.zeros(rows, GH, **f32)
            c_scratch = torch.zeros(rows, H, **f32) if lstm else None
            Gm.gemm(view(hb, t), T * H, False, w, H, False, rows, GH, H, Gm.EPI_F32, gh, GH, bias=b, status=status)
            C().rnn_cell_fwd(rows, H, lstm, view(gi_buf, t), T * GH, gh, GH, view(h_buf, t), T * H, *c_in, None, 0,
                             hout_bf, H, c_scratch, H, done, view(nh, t + 1), T * H, view(hb, t + 1), T * H, *c_next,
                             save, S * H)
        torch.cuda.synchronize()
        outs[fused] = (hout_bf.float(), nh[:, t + 1], hb[:, t + 1].float(), save, nc[:, t + 1] if lstm else None,
                       hb[:, t].float(), hb[:, t - 1].float())
    assert int(status[0]) == 0
    for a_, b_ in zip(outs[True], outs[False]):
        if a_ is not None:
            torch.testing.assert_close(a_, b_, rtol=1e-5, atol=1e-5)
    # against fp32 PyTorch on the same bf16 operands
    gh_ref = hbf_buf[:, t].float() @ w.float().T + b
    ref_h, ref_c = _step_ref(lstm, gi_buf[:, t], gh_ref, h_buf[:, t], c_buf[:, t] if lstm else None)
    keep = (1 - done)[:, None]
    torch.testing.assert_close(outs[True][1], ref_h * keep, rtol=1e-4, atol=1e-4)
    if lstm:
        torch.testing.assert_close(outs[True][4], ref_c * keep, rtol=1e-4, atol=1e-4)
    # the input slot and the slot before it are untouched
    torch.testing.assert_close(outs[True][5], hbf_buf[:, t].float())
    torch.testing.assert_close(outs[True][6], hbf_buf[:, t - 1].float())
