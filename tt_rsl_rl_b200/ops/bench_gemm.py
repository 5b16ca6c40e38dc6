"""Micro-benchmark of the MLP GEMMs on the benchmark model's shapes (forward bias + ELU and data gradient with ELU'
and column sums) for one minibatch of ``--rows`` rows.

Run ``python -m tt_rsl_rl_b200.ops.bench_gemm`` and again with ``RLB_GEMM_WIDE=0`` / ``RLB_GEMM_WIDE=1`` in the
environment to compare the two CTA layouts of the bf16-output epilogues; prints one JSON line of microseconds per
launch (CUDA events around ``--iters`` launches after 3 warm-up launches) and the achieved bandwidth. The shapes are
those of ``rsl_rl/modules/mlp.py:16-95`` in the benchmark model.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from . import gemm as G


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=393216)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    torch.manual_seed(0)
    B, dev = args.rows, "cuda"

    def bf(*s):
        return (torch.randn(*s, device=dev) * 0.5).to(torch.bfloat16)

    out = {"rows": B, "layout": os.environ.get("RLB_GEMM_WIDE", "auto")}

    def timeit(name, fn, nbytes):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1000 / args.iters
        out[name] = {"us": round(us, 1), "TB/s": round(nbytes / us / 1e6, 2)}

    for K, N in ((96, 512), (512, 256), (256, 128)):
        x, w = bf(B, K), bf(N, K)
        bias = torch.randn(N, device=dev)
        y = torch.empty(B, N, device=dev, dtype=torch.bfloat16)
        timeit(f"forward {K}->{N}", lambda: G.gemm(x, K, False, w, K, False, B, N, K, G.EPI_BIAS_ELU_BF16, y, N,
                                                   bias=bias), 2 * B * (K + N))
    for Kout, Nin in ((256, 512), (128, 256), (32, 128)):
        dz, w, h = bf(B, Kout), bf(Kout, Nin), bf(B, Nin)
        y = torch.empty(B, Nin, device=dev, dtype=torch.bfloat16)
        cs = torch.empty(G.colsum_rows(dev), Nin, device=dev)
        timeit(f"data gradient {Kout}->{Nin}",
               lambda: G.gemm(dz, Kout, False, w, Nin, True, B, Nin, Kout, G.EPI_DGRAD_ELU, y, Nin, aux=h,
                              ld_aux=Nin, colsum=cs), 2 * B * (Kout + 2 * Nin))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
