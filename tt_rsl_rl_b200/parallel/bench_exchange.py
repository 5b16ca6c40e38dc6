"""Micro-benchmark of the fused gradient exchange + clip + adaptive-LR + Adam kernel (one PPO optimizer step).

Run ``python -m torch.distributed.run --nproc-per-node N -m tt_rsl_rl_b200.parallel.bench_exchange`` (or plainly for
one GPU). The parameter set has the shapes of the benchmark actor-critic (obs 96/99, 29 actions, [512, 256, 128]), so
the exchange moves the same ~1.73 MB of fp32 gradients per rank as a PPO minibatch step.

Reported (rank 0, one JSON line): device time per step (CUDA events around a CUDA graph of K back-to-back launches,
max over ranks; the eager per-launch time is reported as well),
the roofline time = max(local HBM bytes / measured HBM bandwidth, peer bytes / 770 GB/s per direction), the achieved
fraction of that roofline, and for comparison the time of the baseline path (NCCL all-reduce of the flat gradient +
two clip_grad_norm_ + torch.optim.Adam, as upstream rsl_rl does it: ``rsl_rl/algorithms/ppo.py:304-311`` with the
bucketed all-reduce of ``rsl_rl/utils/utils.py:345-392``).
"""

from __future__ import annotations

import argparse
import json
import os

import torch

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool's B200 nodes
HBM_FALLBACK_GBS = 6650.0


def _hbm_gbs() -> float:
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return HBM_FALLBACK_GBS


def param_shapes() -> list[tuple[tuple[int, ...], int]]:
    """(shape, group) of the benchmark actor (group 0, with std) and critic (group 1) parameters."""
    shapes = [((29,), 0)]
    dims_a = [96, 512, 256, 128, 29]
    dims_c = [99, 512, 256, 128, 1]
    for dims, g in ((dims_a, 0), (dims_c, 1)):
        for i in range(len(dims) - 1):
            shapes.append(((dims[i + 1], dims[i]), g))
            shapes.append(((dims[i + 1],), g))
    return shapes


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--exchange", choices=["one_shot", "two_shot"], default="one_shot",
                    help="one-shot: every rank sums every element; two-shot: reduce-scatter, then owner reads")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=datetime.timedelta(seconds=120))
    from tt_rsl_rl_b200.ops import ext

    C = ext()
    shapes = param_shapes()
    offsets, off = [], 0
    for shape, _ in shapes:
        offsets.append(off)
        off += int(torch.Size(shape).numel())
    n = off
    n_ex = (n + 4 + 3) // 4 * 4
    torch.manual_seed(0)
    flat = torch.randn(n, device=dev) * 0.05
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    grads = torch.zeros(n_ex, device=dev)
    shadows = [torch.zeros(s[0], (s[1] + 7) // 8 * 8, dtype=torch.bfloat16, device=dev) if len(s) == 2 else None
               for s, _ in shapes]
    comm = None
    if world > 1:
        from tt_rsl_rl_b200.parallel import PeerExchange

        comm = PeerExchange.create(n_ex, 4096, rank=rank, world=world, device=dev, timeout_ms=10000)
        send = comm.send
    else:
        b = torch.zeros(n_ex, device=dev)
        send = [b, b]
    torch.manual_seed(1 + rank)
    for sb in send:
        sb[:n].copy_(torch.randn(n, device=dev) * 0.01)
        sb[n + 3] = 0.01
    n_actor = sum(int(torch.Size(s).numel()) for s, g in shapes if g == 0)
    tens, chunks, nch = C.make_adam_plan(
        offsets + [n], [int(torch.Size(s).numel()) for s, _ in shapes] + [4], [g for _, g in shapes] + [-1],
        [s[0] if len(s) == 2 else 1 for s, _ in shapes] + [1], [s[1] if len(s) == 2 else s[0] for s, _ in shapes] + [4],
        shadows + [None], [sh.shape[1] if sh is not None else 0 for sh in shadows] + [0], flat)
    grid = C.adam_grid(local)
    lr = torch.tensor([1e-3, 1e-3], device=dev)
    step = torch.zeros(2, dtype=torch.int64, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    norm_partial = torch.zeros(grid * 4, device=dev)
    barrier = torch.zeros(4, dtype=torch.int32, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)

    two_shot = args.exchange == "two_shot"

    def fused_step():
        C.adam_step(flat, send[0], send[1], grads, m, v, tens, chunks, nch, [1.0, 1.0], [0.9, 0.9], [0.999, 0.999],
                    [1e-8, 1e-8], [0, 0], lr, None, step, True, grads[n + 3 : n + 4], 0.01, 1e-5, 1e-2, world, rank,
                    None if comm is None else comm.peer_send, None if comm is None else comm.peer_flags, epoch,
                    10 * 10**9, norm_partial, barrier, status, None, grid, [0, n_actor, n_actor, n], n_ex,
                    comm.peer_reduced if (comm is not None and two_shot) else None, n + 3)

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1000.0 / steps
        if world > 1:
            t = torch.tensor([us], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            us = float(t.item())
        return us

    # device time of the fused kernel: K launches captured in one CUDA graph (as in the training step, whose update
    # is a graph replay), so host launch overhead is excluded
    for _ in range(args.warmup):
        fused_step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(args.steps):
                fused_step()
    torch.cuda.current_stream(dev).wait_stream(side)
    fused_us = timed(graph.replay, 1, 1) / args.steps
    eager_us = timed(fused_step, args.steps, args.warmup)
    assert int(status[0].item()) == 0, status.tolist()

    # baseline: NCCL all-reduce of the flat gradient + per-model clip + torch Adam (upstream's sequence)
    params = [torch.nn.Parameter(flat[o : o + int(torch.Size(s).numel())].view(s).clone()) for (s, _), o in
              zip(shapes, offsets)]
    for p in params:
        p.grad = torch.randn_like(p) * 0.01
    opt = torch.optim.Adam(params, lr=1e-3)
    groups = [[p for p, (_, g) in zip(params, shapes) if g == k] for k in (0, 1)]
    flat_grad = torch.zeros(n, device=dev)

    def baseline_step():
        if world > 1:
            torch.distributed.all_reduce(flat_grad)
            flat_grad.div_(world)
        torch.nn.utils.clip_grad_norm_(groups[0], 1.0)
        torch.nn.utils.clip_grad_norm_(groups[1], 1.0)
        opt.step()

    base_us = timed(baseline_step, min(args.steps, 100), args.warmup)

    hbm = _hbm_gbs()
    local_bytes = 4 * n * 9 + 2 * sum(sh.numel() for sh in shadows if sh is not None)  # send,g,p,m,v rd/wr + shadows
    peer_bytes = 4 * n_ex * (world - 1) if not two_shot else int(2 * 4 * n_ex * (world - 1) / world)
    roof_us = max(local_bytes / (hbm * 1e3), peer_bytes / (NVLINK_GBS * 1e3))
    # lower bound of any all-reduce algorithm: 2 (N - 1) / N of the vector crosses the links per rank
    min_bytes = 2.0 * (world - 1) / world * 4 * n_ex
    roof_min_us = max(local_bytes / (hbm * 1e3), min_bytes / (NVLINK_GBS * 1e3))
    if rank == 0:
        print(json.dumps({
            "kernel": "fused exchange + clip + adaptive LR + Adam", "exchange": args.exchange, "world": world,
            "params": n,
            "grad_bytes_per_rank": 4 * n_ex, "fused_us": fused_us, "fused_eager_launch_us": eager_us,
            "roofline_us": roof_us,
            "roofline_fraction": roof_us / fused_us, "peer_bytes_per_rank": peer_bytes, "local_hbm_bytes": local_bytes,
            "roofline_us_min_allreduce_bytes": roof_min_us, "roofline_fraction_min_allreduce_bytes": roof_min_us / fused_us,
            "baseline_nccl_torch_adam_us": base_us, "speedup_vs_baseline": base_us / fused_us,
            "hbm_gbs": hbm, "nvlink_gbs": NVLINK_GBS,
        }))
    if comm is not None:
        comm.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
