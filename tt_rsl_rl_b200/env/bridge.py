"""Remote environment bridge: run the learner here and the simulator in another process or on another host.

Transport: ZeroMQ REQ/REP. A message is a multipart list ``[header, buffer_0, buffer_1, ...]``; ``header`` is UTF-8
JSON ``{"op": ..., "tensors": [{"key": k, "dtype": d, "shape": s}, ...], ...}`` and ``buffer_i`` holds the raw
little-endian bytes of tensor ``i`` (C order). Tensor parts are sent from the tensors' own memory and received
without an intermediate copy (ZeroMQ's zero-copy mode; it copies parts below its threshold itself), so a tensor is
copied once on each side. Keys are ``"obs/<group>"``, ``"rewards"``, ``"dones"``,
``"actions"``, ``"time_outs"``, ``"episode_length_buf"``; scalar logging extras travel in the header (``"log"``).

Operations: ``info`` (protocol version, sizes, groups and the host's agent configuration if it has one),
``get_observations``, ``reset`` (when the environment has one), ``step`` (actions in, transition out, episode lengths
included), ``set_episode_length_buf`` (the runner's random start lengths reach the simulator), ``close``. The client
keeps per-operation call counts, seconds and bytes (``RemoteVecEnv.stats``).
A handler error is answered with ``{"op": "error", "message": ...}`` and the server keeps serving; the client turns it
into :class:`RemoteEnvError`. A client whose request gets no reply within ``timeout_ms`` raises
:class:`RemoteEnvTimeoutError` instead of hanging (and rebuilds its socket, as a REQ socket cannot send twice).

The reference plugin's bridge has the same roles (``rsl_rl_tt/bridge/client.py:47-132``, ``server.py:62-154``).
"""

from __future__ import annotations

import json
import threading
import time

import numpy as np
import torch

from ..utils.tensordict import TensorDict
from .vec_env import VecEnv

PROTOCOL_VERSION = 1

_DTYPES = {"float32": torch.float32, "float64": torch.float64, "int64": torch.int64, "int32": torch.int32,
           "uint8": torch.uint8, "bool": torch.bool}
# wire dtype name -> numpy dtype of the frame (booleans travel as bytes)
_NP_DTYPES = {"float32": np.float32, "float64": np.float64, "int64": np.int64, "int32": np.int32, "uint8": np.uint8,
              "bool": np.uint8}


class RemoteEnvError(RuntimeError):
    """The environment server answered a request with an error."""


class RemoteEnvTimeoutError(TimeoutError):
    """The environment server did not answer within the client's timeout."""


def pack(header: dict, tensors: dict[str, torch.Tensor]) -> list:
    """Encode a header and named tensors as a multipart message: the header's bytes, then one buffer per tensor that
    views the (CPU, contiguous) tensor's memory, so a zero-copy send moves it without an intermediate bytes copy."""
    meta, frames = [], []
    for key, t in tensors.items():
        a = t.detach().to("cpu")
        if a.dtype == torch.bool:
            a = a.to(torch.uint8)
        a = a.contiguous()
        meta.append({"key": key, "dtype": str(t.dtype).replace("torch.", ""), "shape": list(a.shape)})
        frames.append(memoryview(a.numpy()).cast("B"))
    return [json.dumps(dict(header, tensors=meta)).encode()] + frames


def _buffer(frame):
    """The bytes of a received part: a ``zmq.Frame`` (zero-copy receive) or any bytes-like object."""
    return frame.buffer if hasattr(frame, "buffer") else frame


def unpack(frames: list) -> tuple[dict, dict[str, torch.Tensor]]:
    """Decode a multipart message into its header and named CPU tensors (one copy out of the message buffers)."""
    header = json.loads(bytes(_buffer(frames[0])).decode())
    out = {}
    for meta, frame in zip(header.get("tensors", []), frames[1:]):
        dt = _DTYPES[meta["dtype"]]
        arr = np.frombuffer(_buffer(frame), dtype=_NP_DTYPES[meta["dtype"]]).reshape(meta["shape"])
        t = torch.from_numpy(arr.copy())
        out[meta["key"]] = t.to(torch.bool) if dt == torch.bool else t
    return header, out


def _transition(env, obs, rewards=None, dones=None, extras=None) -> tuple[dict, dict]:
    tensors = {f"obs/{g}": obs[g] for g in obs.keys()}
    header = {"op": "ok"}
    if rewards is not None:
        tensors["rewards"] = rewards.reshape(-1).float()
        tensors["dones"] = dones.reshape(-1).float()
        tensors["episode_length_buf"] = env.episode_length_buf
        extras = extras or {}
        if "time_outs" in extras:
            tensors["time_outs"] = extras["time_outs"].reshape(-1).float()
        log = extras.get("log") or extras.get("episode") or {}
        header["log"] = {k: float(v.float().mean()) if isinstance(v, torch.Tensor) else float(v) for k, v in log.items()}
    return header, tensors


class EnvServer:
    """Serves a :class:`VecEnv` on a ZeroMQ REP socket until a ``close`` request (or :meth:`stop`)."""

    def __init__(self, env, address: str = "tcp://127.0.0.1:5555", poll_ms: int = 100,
                 agent_cfg: dict | None = None) -> None:
        import zmq

        self.env = env
        # the host's training configuration (JSON-serialisable), handed to the learner with "info"
        self.agent_cfg = None if agent_cfg is None else json.loads(json.dumps(agent_cfg, default=repr))
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.REP)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.sock.bind(address)
        self.address = self.sock.getsockopt_string(zmq.LAST_ENDPOINT)
        self.poll_ms = poll_ms
        self._stop = threading.Event()
        self.errors = 0

    def _handle(self, header: dict, tensors: dict) -> tuple[dict, dict]:
        env, op = self.env, header.get("op")
        if op == "info":
            obs = env.get_observations()
            groups = {g: list(obs[g].shape[1:]) for g in obs.keys()}
            return {"op": "ok", "protocol": PROTOCOL_VERSION, "num_envs": env.num_envs,
                    "num_actions": env.num_actions, "max_episode_length": int(env.max_episode_length),
                    "groups": groups, "step_dt": float(getattr(env, "step_dt", 0.0)), "agent_cfg": self.agent_cfg,
                    "has_reset": callable(getattr(env, "reset", None))}, {"episode_length_buf": env.episode_length_buf}
        if op == "get_observations":
            return _transition(env, env.get_observations())
        if op == "reset":
            reset = getattr(env, "reset", None)
            if not callable(reset):
                raise ValueError("the environment has no reset()")
            out = reset()
            obs, extras = out if isinstance(out, tuple) else (out, {})
            header, tensors = _transition(env, obs)
            log = (extras or {}).get("log") or {}
            header["log"] = {k: float(v.float().mean()) if isinstance(v, torch.Tensor) else float(v) for k, v in log.items()}
            tensors["episode_length_buf"] = env.episode_length_buf
            return header, tensors
        if op == "set_episode_length_buf":
            buf = tensors["episode_length_buf"]
            if buf.shape != (env.num_envs,):
                raise ValueError(f"episode_length_buf must have shape ({env.num_envs},), got {tuple(buf.shape)}")
            env.episode_length_buf = buf.to(dtype=torch.long, device=env.episode_length_buf.device)
            return {"op": "ok"}, {}
        if op == "step":
            actions = tensors["actions"]
            if actions.shape != (env.num_envs, env.num_actions):
                raise ValueError(f"actions must have shape {(env.num_envs, env.num_actions)}, got {tuple(actions.shape)}")
            obs, rew, dones, extras = env.step(actions.to(env.device))
            return _transition(env, obs, rew, dones, extras)
        if op == "close":
            self._stop.set()
            return {"op": "ok"}, {}
        raise ValueError(f"unknown op {op!r}")

    def serve(self) -> None:
        import zmq

        poller = zmq.Poller()
        poller.register(self.sock, zmq.POLLIN)
        while not self._stop.is_set():
            if not dict(poller.poll(self.poll_ms)):
                continue
            frames = self.sock.recv_multipart(copy=False)
            try:
                header, tensors = unpack(frames)
                reply = pack(*self._handle(header, tensors))
            except Exception as exc:  # the server survives handler errors and reports them
                self.errors += 1
                reply = pack({"op": "error", "message": f"{type(exc).__name__}: {exc}"}, {})
            self.sock.send_multipart(reply, copy=False)
        self.sock.close(0)

    def serve_in_thread(self) -> threading.Thread:
        th = threading.Thread(target=self.serve, daemon=True)
        th.start()
        return th

    def stop(self) -> None:
        self._stop.set()


class BridgeStats:
    """Per-operation call count, seconds and payload bytes seen by a client."""

    def __init__(self) -> None:
        self.calls: dict[str, int] = {}
        self.seconds: dict[str, float] = {}
        self.sent_bytes = 0
        self.received_bytes = 0

    def add(self, op: str, seconds: float, sent: int, received: int) -> None:
        self.calls[op] = self.calls.get(op, 0) + 1
        self.seconds[op] = self.seconds.get(op, 0.0) + seconds
        self.sent_bytes += sent
        self.received_bytes += received

    def summary(self) -> dict:
        return {op: {"calls": n, "ms_per_call": 1e3 * self.seconds[op] / n} for op, n in self.calls.items()} | {
            "sent_bytes": self.sent_bytes, "received_bytes": self.received_bytes}


def _nbytes(frames) -> int:
    return sum(len(_buffer(f)) if not isinstance(f, memoryview) else f.nbytes for f in frames)


class RemoteVecEnv(VecEnv):
    """A :class:`VecEnv` whose simulator runs behind an :class:`EnvServer`."""

    def __init__(self, address: str, device: str | torch.device = "cpu", timeout_ms: int = 30000) -> None:
        import zmq

        self.address = address
        self.device = torch.device(device)
        self.timeout_ms = int(timeout_ms)
        self._zmq = zmq
        self.ctx = zmq.Context.instance()
        self.stats = BridgeStats()
        self._connect()
        info, t = self._request({"op": "info"}, {})
        if info.get("protocol") != PROTOCOL_VERSION:
            raise RemoteEnvError(f"the server speaks bridge protocol {info.get('protocol')}, this client "
                                 f"{PROTOCOL_VERSION}")
        self.has_reset = bool(info.get("has_reset", False))
        self.num_envs = int(info["num_envs"])
        self.num_actions = int(info["num_actions"])
        self.max_episode_length = int(info["max_episode_length"])
        self.step_dt = float(info.get("step_dt", 0.0))
        self.groups = info["groups"]
        self.agent_cfg = info.get("agent_cfg")  # the server's training configuration, if it sent one
        self._episode_length_buf = t["episode_length_buf"].to(self.device)
        self.cfg = {"address": address, "num_envs": self.num_envs}

    @property
    def unwrapped(self) -> RemoteVecEnv:
        return self

    def _connect(self) -> None:
        zmq = self._zmq
        self.sock = self.ctx.socket(zmq.REQ)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.sock.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
        self.sock.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
        self.sock.connect(self.address)

    @property
    def episode_length_buf(self) -> torch.Tensor:
        """Episode lengths of the remote environments (refreshed by every step)."""
        return self._episode_length_buf

    @episode_length_buf.setter
    def episode_length_buf(self, value: torch.Tensor) -> None:
        """Set the remote environments' episode lengths (the runner's random start lengths)."""
        value = torch.as_tensor(value, dtype=torch.long).reshape(self.num_envs)
        self._request({"op": "set_episode_length_buf"}, {"episode_length_buf": value})
        self._episode_length_buf = value.to(self.device)

    def _request(self, header: dict, tensors: dict) -> tuple[dict, dict]:
        zmq = self._zmq
        t0 = time.perf_counter()
        try:
            request = pack(header, tensors)
            self.sock.send_multipart(request, copy=False)
            frames = self.sock.recv_multipart(copy=False)
        except zmq.error.Again as exc:
            # a REQ socket that missed its reply cannot send again: rebuild it before reporting
            self.sock.close(0)
            self._connect()
            raise RemoteEnvTimeoutError(
                f"environment server at {self.address} did not answer {header.get('op')!r} within {self.timeout_ms} ms"
            ) from exc
        reply, out = unpack(frames)
        self.stats.add(header.get("op", "?"), time.perf_counter() - t0, _nbytes(request), _nbytes(frames))
        if reply.get("op") == "error":
            raise RemoteEnvError(reply.get("message", "remote error"))
        return reply, out

    def _obs(self, tensors: dict) -> TensorDict:
        groups = {k[4:]: v.to(self.device) for k, v in tensors.items() if k.startswith("obs/")}
        return TensorDict(groups, batch_size=[self.num_envs], device=self.device)

    def get_observations(self):
        _, tensors = self._request({"op": "get_observations"}, {})
        return self._obs(tensors)

    def reset(self):
        """Reset every remote environment (when the server's environment has ``reset()``)."""
        reply, t = self._request({"op": "reset"}, {})
        self._episode_length_buf = t["episode_length_buf"].to(self.device)
        extras = {"log": {k: torch.tensor(v) for k, v in reply["log"].items()}} if reply.get("log") else {}
        return self._obs(t), extras

    def step(self, actions: torch.Tensor):
        reply, t = self._request({"op": "step"}, {"actions": actions.float()})
        obs = self._obs(t)
        rewards = t["rewards"].to(self.device)
        dones = t["dones"].to(self.device)
        self._episode_length_buf = t["episode_length_buf"].to(self.device)
        extras = {}
        if "time_outs" in t:
            extras["time_outs"] = t["time_outs"].to(self.device)
        if reply.get("log"):
            extras["log"] = {k: torch.tensor(v) for k, v in reply["log"].items()}
        return obs, rewards, dones, extras

    def close(self) -> None:
        try:
            self._request({"op": "close"}, {})
        finally:
            self.sock.close(0)


# ---- command line: serve an environment on one host, train against it on another --------------------------------------
def _make_served_env(args):
    if args.local_env:
        from .classic import make_env

        return make_env(args.local_env, args.num_envs, seed=args.seed, device=args.env_device)
    from ..utils.utils import resolve_callable

    return resolve_callable(args.env)(**json.loads(args.env_kwargs or "{}"))


def serve_main(args) -> int:
    """Serve an environment until a client closes it (the environment host's side)."""
    from .agent_cfg import load_agent_cfg

    env = _make_served_env(args)
    agent_cfg = load_agent_cfg(args.agent_cfg) if args.agent_cfg else None
    if agent_cfg is None and args.local_env:
        from ..testing.reference import train_cfg

        agent_cfg = train_cfg(args.local_env, logger=None)  # the test environment's own run spec
    server = EnvServer(env, args.address, agent_cfg=agent_cfg)
    print(json.dumps({"serving": server.address, "num_envs": int(env.num_envs)}), flush=True)
    server.serve()
    return 0


def train_main(args) -> int:
    """Train against a served environment with the server's (or a saved) agent configuration."""
    from ..runners import OnPolicyRunner
    from .agent_cfg import b200_agent_cfg, load_agent_cfg

    env = RemoteVecEnv(args.address, device=args.device, timeout_ms=args.timeout_ms)
    try:
        agent_cfg = load_agent_cfg(args.agent_cfg) if args.agent_cfg else env.agent_cfg
        if agent_cfg is None:
            raise SystemExit("the server sent no agent configuration; give one with --agent-cfg")
        cfg = b200_agent_cfg(agent_cfg, device=args.device, engine=args.engine, csv_log=True)
        runner = OnPolicyRunner(env, cfg, log_dir=args.log_dir, device=cfg["device"])
        if args.resume:
            runner.resume_latest()
        runner.learn(args.iterations, init_at_random_ep_len=True)
        print(json.dumps({"iterations": args.iterations, "log_dir": args.log_dir, "bridge": env.stats.summary()}))
    finally:
        env.close()
    return 0


def main(argv=None) -> int:
    """``serve`` on the environment host, ``train`` on the learner host::

        python -m tt_rsl_rl_b200.env.bridge serve --local-env tracking12 --num-envs 2048 --address tcp://*:5555
        python -m tt_rsl_rl_b200.env.bridge serve --env my_pkg.envs:make --env-kwargs '{"num_envs": 4096}' \\
            --agent-cfg params/agent.yaml --address tcp://*:5555
        python -m tt_rsl_rl_b200.env.bridge train --address tcp://env-host:5555 --iterations 300 --log-dir logs/run

    The reference plugin splits the same roles over two scripts (``scripts/isaac_env_server.py``,
    ``scripts/train_isaac.py``)."""
    import argparse

    ap = argparse.ArgumentParser(prog="python -m tt_rsl_rl_b200.env.bridge", description=main.__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("serve", help="serve an environment")
    s.add_argument("--address", default="tcp://127.0.0.1:5555")
    s.add_argument("--local-env", default=None, help="a seeded test environment of this package")
    s.add_argument("--env", default=None, help="'module:callable' returning a VecEnv")
    s.add_argument("--env-kwargs", default=None, help="JSON keyword arguments of --env")
    s.add_argument("--num-envs", type=int, default=1024)
    s.add_argument("--seed", type=int, default=0)
    s.add_argument("--env-device", default="cpu")
    s.add_argument("--agent-cfg", default=None, help="JSON / YAML agent configuration handed to the learner")
    t = sub.add_parser("train", help="train against a served environment")
    t.add_argument("--address", required=True)
    t.add_argument("--iterations", type=int, default=100)
    t.add_argument("--log-dir", default=None)
    t.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    t.add_argument("--engine", default="auto", choices=("auto", "torch", "cuda"))
    t.add_argument("--agent-cfg", default=None, help="override the server's agent configuration")
    t.add_argument("--timeout-ms", type=int, default=60_000)
    t.add_argument("--resume", action="store_true", help="continue from the newest checkpoint in --log-dir")
    args = ap.parse_args(argv)
    if args.cmd == "serve":
        if bool(args.local_env) == bool(args.env):
            ap.error("serve needs exactly one of --local-env and --env")
        return serve_main(args)
    return train_main(args)


if __name__ == "__main__":
    raise SystemExit(main())
