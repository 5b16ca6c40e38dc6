"""Micro-benchmark of one recurrent training step (GRU / LSTM) of the fused recurrent path.

Run ``python -m tt_rsl_rl_b200.ops.bench_rnn_step`` on one GPU. The shapes are those of a minibatch step of the
benchmark's recurrent configuration: 4,096 environments, hidden size 256, 24 steps stored env-major
(``[env, T, width]``, the layout of ``engine/recurrent_engine.py``). Every launch works on the next step slot, so inputs
and outputs come from and go to DRAM as in training (the buffers total well over the 126 MB L2).

Reported (one JSON line, microseconds per step, CUDA events around a CUDA graph of 20 back-to-back launches after
warm-up):

* forward: the hidden GEMM ``gh = h W_hh^T + b_hh`` (fp32 out), the cell kernel, both in sequence, and the fused step
  (the GEMM with the cell in its epilogue, ``rnn_step_fused``);
* backward: the cell backward kernel (gate gradients, recurrent gradients, bias column sums) and ``dh = dgh W_hh``.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import ext
from . import gemm as Gm


def _time(fn, n: int = 200) -> float:
    for _ in range(10):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(20):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n // 20):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / n


def bench(lstm: bool, rows: int = 4096, H: int = 256, T: int = 24, case_only: bool = False) -> dict[str, float]:
    C = ext()
    G, S = (4, 5) if lstm else (3, 4)
    GH = G * H
    f32 = dict(device="cuda", dtype=torch.float32)
    hb = torch.randn(rows, T, H, **f32).bfloat16()
    hf = torch.randn(rows, T, H, **f32)
    cf = torch.randn(rows, T, H, **f32) if lstm else None
    gi = torch.randn(rows, T, GH, **f32)
    w = (torch.randn(GH, H, **f32) / H**0.5).bfloat16()
    b = torch.randn(GH, **f32)
    done = (torch.rand(rows, device="cuda") < 0.01).float()
    save = torch.zeros(rows, T, S * H, **f32)
    hout = torch.zeros(rows, T, H, device="cuda", dtype=torch.bfloat16)
    gh = torch.zeros(rows, GH, **f32)
    c_scratch = torch.zeros(rows, H, **f32) if lstm else None
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    dh_head = torch.randn(rows, T, H, **f32)
    dgi = torch.zeros(rows, T, GH, device="cuda", dtype=torch.bfloat16)
    dgh = dgi if lstm else torch.zeros(rows, T, GH, device="cuda", dtype=torch.bfloat16)
    dh_direct = [torch.randn(rows, H, **f32) for _ in range(2)]
    dh_gemm = [torch.randn(rows, H, **f32) for _ in range(2)]
    dc = [torch.randn(rows, H, **f32) for _ in range(2)] if lstm else [None, None]
    nb = C.rnn_bwd_blocks(rows)
    cs_gi = torch.zeros(nb, GH, **f32)
    cs_gh = None if lstm else torch.zeros(nb, GH, **f32)

    def view(buf, t):
        return buf.view(-1)[t * buf.shape[2] :]

    slot = [0]

    def step() -> int:  # a new step slot every launch
        t = slot[0]
        slot[0] = (t + 1) % (T - 1)
        return t

    def states(t):
        if not lstm:
            return (None, 0), (None, 0)
        return (view(cf, t), T * H), (view(cf, t + 1), T * H)

    def gemm(t):
        Gm.gemm(view(hb, t), T * H, False, w, H, False, rows, GH, H, Gm.EPI_F32, gh, GH, bias=b, status=status)

    def cell(t):
        c_in, c_next = states(t)
        C.rnn_cell_fwd(rows, H, lstm, view(gi, t), T * GH, gh, GH, view(hf, t), T * H, *c_in, None, 0, view(hout, t),
                       T * H, c_scratch, H, done, view(hf, t + 1), T * H, view(hb, t + 1), T * H, *c_next,
                       view(save, t), T * S * H)

    def fused(t):
        c_in, c_next = states(t)
        C.rnn_step_fused(rows, H, lstm, view(hb, t), T * H, w, H, b, view(gi, t), T * GH, view(hf, t), T * H, *c_in,
                         None, 0, view(hout, t), T * H, None, 0, done, view(hf, t + 1), T * H, view(hb, t + 1), T * H,
                         *c_next, view(save, t), T * S * H, status)

    def cell_bwd(t):
        C.rnn_cell_bwd(rows, H, lstm, view(save, t), T * S * H, None if lstm else view(hf, t), T * H,
                       view(cf, t) if lstm else None, T * H, view(dh_head, t), T * H, None if lstm else dh_direct[1],
                       dh_gemm[1], H, dc[1], H, done, view(dgi, t), T * GH, None if lstm else view(dgh, t), T * GH,
                       dh_direct[0], H, dc[0], H, cs_gi, cs_gh, True)

    def dh(t):
        Gm.gemm(view(dgh, t), T * GH, False, w, H, True, rows, H, GH, Gm.EPI_F32, dh_gemm[0], H, status=status)

    if case_only:  # five fused steps and nothing else (a small case for ncu: capture the fourth)
        for _ in range(5):
            fused(step())
        torch.cuda.synchronize()
        if int(status[0]) != 0:
            raise RuntimeError(f"device status {status.tolist()}")
        return {}
    out = {
        "gemm_us": _time(lambda: gemm(step())),
        "cell_us": _time(lambda: cell(step())),
        "gemm_plus_cell_us": _time(lambda: (lambda t: (gemm(t), cell(t)))(step())),
        "fused_us": _time(lambda: fused(step())),
        "cell_bwd_us": _time(lambda: cell_bwd(step())),
        "dh_gemm_us": _time(lambda: dh(step())),
    }
    torch.cuda.synchronize()
    if int(status[0]) != 0:
        raise RuntimeError(f"device status {status.tolist()}")
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=256)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--ncu-case", choices=["gru", "lstm"], default=None,
                    help="only launch five fused steps of this cell (a small case to capture under ncu)")
    args = ap.parse_args()
    if args.ncu_case:
        bench(args.ncu_case == "lstm", args.rows, args.hidden, args.steps, case_only=True)
        print(json.dumps({"ncu_case": args.ncu_case, "fused_steps": 5}))
        return
    res = {name: bench(name == "lstm", args.rows, args.hidden, args.steps) for name in ("gru", "lstm")}
    res["shape"] = {"rows": args.rows, "hidden": args.hidden, "steps": args.steps}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
