"""Host-side rules of the fused recurrent paths, checked against the PyTorch path's definitions: the window schedule
of recurrent distillation students and the padded-entry count of recurrent RND minibatches."""

import pytest
import torch


def _upstream_windows(epochs, steps, gl):
    """(epoch, step, window, applied) per step as upstream's loop counts them: the loss sum runs across epochs and is
    applied every ``gl`` steps; steps after the last full window are never applied."""
    out, cnt = [], 0
    total = epochs * steps
    for e in range(epochs):
        for t in range(steps):
            cnt += 1
            out.append((e, t, (cnt - 1) // gl, cnt <= total // gl * gl))
    return out


@pytest.mark.parametrize("epochs,steps,gl", [(1, 8, 4), (2, 8, 3), (2, 8, 5), (3, 8, 10), (2, 24, 24), (4, 5, 7),
                                             (1, 3, 1)])
def test_window_segments_follow_the_step_count(epochs, steps, gl):
    from tt_rsl_rl_b200.engine.distillation_engine import window_segments

    segs = window_segments(epochs, steps, gl)
    ref = _upstream_windows(epochs, steps, gl)
    # the segments tile every epoch's steps in order
    flat = [(e, t0 + k) for e, t0, L, *_ in segs for k in range(L)]
    assert flat == [(e, t) for e, t, _, _ in ref]
    i = 0
    for e, t0, L, first, train, apply in segs:
        steps_here = ref[i : i + L]
        i += L
        # one epoch and one window per segment
        assert len({s[0] for s in steps_here}) == 1 and len({s[2] for s in steps_here}) == 1
        window = steps_here[0][2]
        assert first == (i - L == 0 or ref[i - L - 1][2] != window)
        assert train == steps_here[-1][3]
        last_of_window = i == len(ref) or ref[i][2] != window
        assert apply == (train and last_of_window)
    assert sum(a for *_, a in segs) == epochs * steps // gl


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_rnd_padded_entries_formula(seed):
    """The zero-padded entries of a recurrent minibatch (environments lo .. lo + Be - 1) equal T times the dones
    before the last step in that range, as rnn_pad_entries computes them."""
    from tt_rsl_rl_b200.utils.utils import split_and_pad_trajectories

    g = torch.Generator().manual_seed(seed)
    T, N, M = 12, 40, 4
    dones = (torch.rand(T, N, 1, generator=g) < 0.15).float()
    x = torch.arange(T * N, dtype=torch.float32).reshape(T, N, 1) + 1.0
    padded, masks = split_and_pad_trajectories(x, dones)
    assert padded.shape[0] == T
    first = 0
    for i in range(M):
        lo, hi = i * N // M, (i + 1) * N // M
        last_was_done = torch.zeros(T, N, dtype=torch.bool)
        last_was_done[1:] = dones[:-1, :, 0].bool()
        last_was_done[0] = True
        n_traj = int(last_was_done[:, lo:hi].sum())
        block = masks[:, first : first + n_traj]
        first += n_traj
        assert int(block.sum()) == (hi - lo) * T  # every real entry once
        pad = n_traj * T - (hi - lo) * T
        assert pad == T * int(dones[: T - 1, lo:hi].sum())
