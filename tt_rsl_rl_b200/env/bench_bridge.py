"""Round trip and bandwidth of the environment bridge, host only: the server runs in its own process on loopback
and serves a :class:`~tt_rsl_rl_b200.env.null.NullVecEnv`, so only the transport is measured.

One step sends the actions (``num_envs x A`` float32) and returns the observation groups, rewards, dones, time-outs
(float32) and episode lengths (int64). Transports on the same payload:

* ``zmq-tcp`` / ``zmq-ipc``: the bridge (:class:`~tt_rsl_rl_b200.env.bridge.RemoteVecEnv` against
  :class:`~tt_rsl_rl_b200.env.bridge.EnvServer`): JSON header plus raw tensor frames;
* ``zmq-pickle``: ZeroMQ ``send_pyobj`` of the tensors, the naive alternative;
* ``raw-tcp``: a plain TCP socket carrying the same bytes with a length prefix and no encoding, the loopback floor;
* ``reference-zmq-tcp``: the reference plugin's own bridge (``rsl_rl_tt/bridge``, importable from an install of the
  reference) serving the same environment, for a same-machine comparison (its payload differs slightly: it sends
  dones as bytes and no episode lengths; the bytes it moved are reported).

::

    python -m tt_rsl_rl_b200.env.bench_bridge --envs 1024 4096 16384 --steps 200

The reference plugin measures the same comparison (``scripts/bench_bridge.py``).
"""

from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import shutil
import socket
import statistics
import struct
import tempfile
import time

import torch

SHAPES = {"tracking12": ({"policy": 36, "privileged": 48}, 12), "humanoid": ({"policy": 96, "critic": 99}, 29)}
TRANSPORTS = ("zmq-tcp", "zmq-ipc", "zmq-pickle", "raw-tcp", "reference-zmq-tcp")


def step_bytes(num_envs: int, groups: dict[str, int], num_actions: int) -> tuple[int, int]:
    """(bytes sent, bytes received) per step, payload only."""
    sent = num_envs * num_actions * 4
    received = num_envs * (4 * sum(groups.values()) + 3 * 4 + 8)
    return sent, received


def _null_env(num_envs, shape):
    from .null import NullVecEnv

    groups, A = SHAPES[shape]
    return NullVecEnv(num_envs, groups, A)


def _serve_bridge(address, num_envs, shape, ready):
    from .bridge import EnvServer

    srv = EnvServer(_null_env(num_envs, shape), address)
    ready.put(srv.address)
    srv.serve()


def _serve_pickle(address, num_envs, shape, ready):
    import zmq

    env = _null_env(num_envs, shape)
    sock = zmq.Context.instance().socket(zmq.REP)
    sock.bind(address)
    ready.put(sock.getsockopt_string(zmq.LAST_ENDPOINT))
    while True:
        msg = sock.recv_pyobj()
        if msg is None:
            sock.send_pyobj(None)
            break
        obs, rew, dones, extras = env.step(msg)
        sock.send_pyobj(({k: obs[k] for k in obs.keys()}, rew, dones, extras["time_outs"], env.episode_length_buf))
    sock.close(0)


def _reference_bridge():
    """The reference plugin's bridge package (``rsl_rl_tt.bridge``), from an install of the reference."""
    import importlib

    try:
        return importlib.import_module("rsl_rl_tt.bridge.server"), importlib.import_module("rsl_rl_tt.bridge.client")
    except ImportError:
        import baseline

        if not baseline.reference_available():
            raise
        baseline.add_reference_to_path()
        return importlib.import_module("rsl_rl_tt.bridge.server"), importlib.import_module("rsl_rl_tt.bridge.client")


def _serve_reference(address, num_envs, shape, ready):
    server, _ = _reference_bridge()
    ready.put(address)
    server.serve(_null_env(num_envs, shape), address, log=lambda m: None)


def _recv_exact(conn, n):
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        k = conn.recv_into(view[got:], n - got)
        if k == 0:
            raise ConnectionError("peer closed")
        got += k
    return buf


def _serve_raw(num_envs, shape, ready):
    env = _null_env(num_envs, shape)
    obs = env.get_observations()
    reply = b"".join([*(obs[k].numpy().tobytes() for k in obs.keys()), env._rewards.numpy().tobytes(),
                      env._dones.numpy().tobytes(), env._extras["time_outs"].numpy().tobytes(),
                      env.episode_length_buf.numpy().tobytes()])
    srv = socket.socket()
    srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    ready.put(srv.getsockname()[1])
    conn, _ = srv.accept()
    conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    while True:
        (n,) = struct.unpack("<Q", _recv_exact(conn, 8))
        if n == 0:
            break
        _recv_exact(conn, n)  # the actions (not used by a null environment)
        conn.sendall(struct.pack("<Q", len(reply)) + reply)
    conn.close()
    srv.close()


def _time_steps(step, steps: int, warmup: int) -> list[float]:
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        step()
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return times


def measure(transport: str, num_envs: int, steps: int = 200, warmup: int = 20, shape: str = "tracking12") -> dict:
    """Median and p90 round trip of one step over ``transport``; payload bandwidth from the median."""
    groups, A = SHAPES[shape]
    actions = torch.zeros(num_envs, A)
    ctx = mp.get_context("spawn")
    ready = ctx.Queue()
    tmp = tempfile.mkdtemp(prefix="bridge_bench_")
    if transport in ("zmq-tcp", "zmq-ipc", "zmq-pickle"):
        address = f"ipc://{os.path.join(tmp, 'sock')}" if transport == "zmq-ipc" else "tcp://127.0.0.1:*"
        target = _serve_pickle if transport == "zmq-pickle" else _serve_bridge
        proc = ctx.Process(target=target, args=(address, num_envs, shape, ready), daemon=True)
    elif transport == "raw-tcp":
        proc = ctx.Process(target=_serve_raw, args=(num_envs, shape, ready), daemon=True)
    elif transport == "reference-zmq-tcp":
        with socket.socket() as probe:
            probe.bind(("127.0.0.1", 0))
            port = probe.getsockname()[1]
        proc = ctx.Process(target=_serve_reference, args=(f"tcp://127.0.0.1:{port}", num_envs, shape, ready),
                           daemon=True)
    else:
        raise ValueError(f"unknown transport {transport!r}; known: {TRANSPORTS}")
    proc.start()
    try:
        endpoint = ready.get(timeout=120)
        if transport == "raw-tcp":
            conn = socket.create_connection(("127.0.0.1", endpoint))
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            payload = actions.numpy().tobytes()

            def step():
                conn.sendall(struct.pack("<Q", len(payload)) + payload)
                (n,) = struct.unpack("<Q", _recv_exact(conn, 8))
                _recv_exact(conn, n)

            times = _time_steps(step, steps, warmup)
            conn.sendall(struct.pack("<Q", 0))
            conn.close()
        elif transport == "zmq-pickle":
            import zmq

            sock = zmq.Context.instance().socket(zmq.REQ)
            sock.setsockopt(zmq.LINGER, 0)
            sock.connect(endpoint)

            def step():
                sock.send_pyobj(actions)
                sock.recv_pyobj()

            times = _time_steps(step, steps, warmup)
            sock.send_pyobj(None)
            sock.recv_pyobj()
            sock.close(0)
        elif transport == "reference-zmq-tcp":
            _, client = _reference_bridge()
            env = client.RemoteVecEnv(endpoint, timeout_s=60)
            times = _time_steps(lambda: env.step(actions), steps, warmup)
            moved = (env.stats.sent_bytes + env.stats.received_bytes) // max(1, len(env.stats.step_rtt_s))
            env.close()
        else:
            from .bridge import RemoteVecEnv

            env = RemoteVecEnv(endpoint, timeout_ms=60_000)
            times = _time_steps(lambda: env.step(actions), steps, warmup)
            env.close()
    finally:
        proc.join(timeout=10)
        if proc.is_alive():
            proc.terminate()
            proc.join()
        shutil.rmtree(tmp, ignore_errors=True)
    sent, received = step_bytes(num_envs, groups, A)
    if transport == "reference-zmq-tcp":
        sent, received = moved, 0  # measured by the reference client (includes its info / header bytes)
    med = statistics.median(times)
    return {"transport": transport, "num_envs": num_envs, "shape": shape, "steps": steps,
            "ms_per_step": round(med * 1e3, 4), "p90_ms": round(sorted(times)[int(0.9 * (len(times) - 1))] * 1e3, 4),
            "bytes_per_step": sent + received, "mb_per_s": round((sent + received) / med / 1e6, 1),
            "steps_per_s": round(1.0 / med, 1)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--envs", type=int, nargs="+", default=[1024, 4096, 16384])
    ap.add_argument("--transports", nargs="+", choices=TRANSPORTS, default=list(TRANSPORTS))
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--shape", choices=sorted(SHAPES), default="tracking12")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    results = []
    for n in args.envs:
        for t in args.transports:
            res = measure(t, n, args.steps, args.warmup, args.shape)
            print(json.dumps(res), flush=True)
            results.append(res)
    if args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)


if __name__ == "__main__":
    main()
