"""A small TensorDict: a dict of tensors that share leading "batch" dimensions.

rsl_rl passes observations as ``tensordict.TensorDict`` objects (``rsl_rl/env/vec_env.py:45``,
``rsl_rl/storage/rollout_storage.py:142``). The ``tensordict`` package is not part of this image, so the framework ships
the subset of that interface it and user environments need: construction with ``batch_size``/``device``, key access,
batch indexing/slicing (returning views), ``copy_``, ``to``, ``clone``, ``flatten``, ``view``, ``transpose``,
``torch.cat``/``torch.stack`` and ``apply``. If the real package is importable, its objects are accepted everywhere this
class is (the framework only relies on the mapping interface and ``batch_size``).

This module has no dependency on the rest of the package.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, Mapping
from typing import Any

import torch

_TORCH_FUNCTIONS: dict[Callable, Callable] = {}


def _implements(fn: Callable) -> Callable:
    def deco(impl: Callable) -> Callable:
        _TORCH_FUNCTIONS[fn] = impl
        return impl

    return deco


class TensorDict:
    """Mapping from names to tensors whose first ``len(batch_size)`` dimensions equal ``batch_size``."""

    __slots__ = ("_data", "_batch_size", "_device")

    def __init__(
        self,
        source: Mapping[str, torch.Tensor] | None = None,
        batch_size: torch.Size | list[int] | tuple[int, ...] | None = None,
        device: torch.device | str | None = None,
    ) -> None:
        self._data: dict[str, Any] = {}
        self._device = torch.device(device) if device is not None else None
        source = dict(source) if source is not None else {}
        if batch_size is None:
            batch_size = self._infer_batch_size(source)
        self._batch_size = torch.Size(batch_size)
        for key, value in source.items():
            self[key] = value

    # ---- construction helpers -------------------------------------------------------------------------------------
    @staticmethod
    def _infer_batch_size(source: Mapping[str, Any]) -> torch.Size:
        shapes = [v.shape for v in source.values() if isinstance(v, (torch.Tensor, TensorDict))]
        if not shapes:
            return torch.Size([])
        common = []
        for dims in zip(*shapes):
            if all(d == dims[0] for d in dims):
                common.append(dims[0])
            else:
                break
        # leave at least one feature dimension when all tensors have the same full shape
        if all(len(s) == len(common) for s in shapes) and common:
            common = common[:-1]
        return torch.Size(common)

    @classmethod
    def _from_parts(cls, data: dict[str, Any], batch_size: torch.Size, device: torch.device | None) -> TensorDict:
        out = cls.__new__(cls)
        out._data = data
        out._batch_size = torch.Size(batch_size)
        out._device = device
        return out

    # ---- mapping interface ----------------------------------------------------------------------------------------
    def keys(self):
        return self._data.keys()

    def values(self):
        return self._data.values()

    def items(self):
        return self._data.items()

    def __iter__(self) -> Iterator[str]:
        return iter(self._data)

    def __len__(self) -> int:
        return self._batch_size[0] if len(self._batch_size) else 0

    def __contains__(self, key: object) -> bool:
        return key in self._data

    def get(self, key: str, default: Any = None) -> Any:
        return self._data.get(key, default)

    def __getitem__(self, index: Any) -> Any:
        if isinstance(index, str):
            return self._data[index]
        if isinstance(index, tuple) and index and all(isinstance(i, str) for i in index):
            out: Any = self
            for key in index:
                out = out[key]
            return out
        return self._index(index)

    def __setitem__(self, index: Any, value: Any) -> None:
        if isinstance(index, str):
            if isinstance(value, (torch.Tensor, TensorDict)):
                if tuple(value.shape[: len(self._batch_size)]) != tuple(self._batch_size):
                    raise ValueError(
                        f"Entry '{index}' has shape {tuple(value.shape)} which does not start with batch size "
                        f"{tuple(self._batch_size)}"
                    )
                if self._device is not None and value.device != self._device:
                    value = value.to(self._device)
            self._data[index] = value
            return
        # batch-indexed assignment: td[idx] = other_td
        if not isinstance(value, (TensorDict, Mapping)):
            raise TypeError("Batch-indexed assignment expects a TensorDict")
        for key, tensor in self._data.items():
            tensor[index] = value[key]

    def __delitem__(self, key: str) -> None:
        del self._data[key]

    def update(self, other: Mapping[str, Any]) -> TensorDict:
        for key, value in other.items():
            self[key] = value
        return self

    def set(self, key: str, value: Any) -> TensorDict:
        self[key] = value
        return self

    def select(self, *keys: str) -> TensorDict:
        return TensorDict._from_parts({k: self._data[k] for k in keys}, self._batch_size, self._device)

    def exclude(self, *keys: str) -> TensorDict:
        return TensorDict._from_parts(
            {k: v for k, v in self._data.items() if k not in keys}, self._batch_size, self._device
        )

    # ---- properties -----------------------------------------------------------------------------------------------
    @property
    def batch_size(self) -> torch.Size:
        return self._batch_size

    @batch_size.setter
    def batch_size(self, value: Any) -> None:
        self._batch_size = torch.Size(value)

    @property
    def shape(self) -> torch.Size:
        return self._batch_size

    @property
    def batch_dims(self) -> int:
        return len(self._batch_size)

    @property
    def device(self) -> torch.device | None:
        if self._device is not None:
            return self._device
        devices = {v.device for v in self._data.values()}
        return devices.pop() if len(devices) == 1 else None

    def numel(self) -> int:
        n = 1
        for d in self._batch_size:
            n *= d
        return n

    def dim(self) -> int:
        return len(self._batch_size)

    def ndimension(self) -> int:
        return self.dim()

    def size(self, dim: int | None = None):
        return self._batch_size if dim is None else self._batch_size[dim]

    def is_empty(self) -> bool:
        return len(self._data) == 0

    # ---- elementwise application ----------------------------------------------------------------------------------
    def apply(self, fn: Callable[[torch.Tensor], torch.Tensor], batch_size: Any = None,
              device: torch.device | str | None = None) -> TensorDict:
        data = {k: (v.apply(fn) if isinstance(v, TensorDict) else fn(v)) for k, v in self._data.items()}
        if batch_size is None:
            batch_size = self._infer_leading(data, len(self._batch_size))
        dev = torch.device(device) if device is not None else self._device
        return TensorDict._from_parts(data, torch.Size(batch_size), dev)

    @staticmethod
    def _infer_leading(data: dict[str, Any], nbatch: int) -> torch.Size:
        for v in data.values():
            return torch.Size(v.shape[:nbatch])
        return torch.Size([])

    def _index(self, index: Any) -> TensorDict:
        data = {k: v[index] for k, v in self._data.items()}
        if data:
            first_key = next(iter(self._data))
            first_old = self._data[first_key]
            first_new = data[first_key]
            feat = first_old.dim() - len(self._batch_size)
            new_batch = first_new.shape[: first_new.dim() - feat]
        else:
            probe = torch.empty(self._batch_size)
            idx = index.cpu() if isinstance(index, torch.Tensor) else index
            new_batch = probe[idx].shape
        return TensorDict._from_parts(data, torch.Size(new_batch), self._device)

    # ---- tensor-like methods --------------------------------------------------------------------------------------
    def to(self, *args: Any, **kwargs: Any) -> TensorDict:
        data = {k: v.to(*args, **kwargs) for k, v in self._data.items()}
        device = None
        for a in list(args) + [kwargs.get("device")]:
            if isinstance(a, (str, torch.device)):
                device = torch.device(a)
        return TensorDict._from_parts(data, self._batch_size, device if device is not None else self._device)

    def cpu(self) -> TensorDict:
        return self.to("cpu")

    def cuda(self, device: int | None = None) -> TensorDict:
        return self.to(torch.device("cuda", device) if device is not None else torch.device("cuda"))

    def clone(self) -> TensorDict:
        return self.apply(lambda t: t.clone(), batch_size=self._batch_size)

    def detach(self) -> TensorDict:
        return self.apply(lambda t: t.detach(), batch_size=self._batch_size)

    def contiguous(self) -> TensorDict:
        return self.apply(lambda t: t.contiguous(), batch_size=self._batch_size)

    def float(self) -> TensorDict:
        return self.apply(lambda t: t.float(), batch_size=self._batch_size)

    def zero_(self) -> TensorDict:
        for v in self._data.values():
            v.zero_()
        return self

    def copy_(self, other: Mapping[str, torch.Tensor], non_blocking: bool = False) -> TensorDict:
        for key, value in self._data.items():
            value.copy_(other[key], non_blocking=non_blocking)
        return self

    def flatten(self, start_dim: int = 0, end_dim: int = -1) -> TensorDict:
        nb = len(self._batch_size)
        s = start_dim % nb
        e = end_dim % nb
        new_batch = list(self._batch_size[:s]) + [int(torch.Size(self._batch_size[s : e + 1]).numel())]
        new_batch += list(self._batch_size[e + 1 :])
        return self.apply(lambda t: t.flatten(s, e), batch_size=new_batch)

    def view(self, *shape: Any) -> TensorDict:
        return self._reshape(shape, copy_ok=False)

    def reshape(self, *shape: Any) -> TensorDict:
        return self._reshape(shape, copy_ok=True)

    def _reshape(self, shape: tuple, copy_ok: bool) -> TensorDict:
        if len(shape) == 1 and isinstance(shape[0], (tuple, list, torch.Size)):
            shape = tuple(shape[0])
        probe = torch.empty(self._batch_size, device="meta").reshape(*shape)
        nb = len(self._batch_size)
        if copy_ok:
            return self.apply(lambda t: t.reshape(*probe.shape, *t.shape[nb:]), batch_size=probe.shape)
        return self.apply(lambda t: t.view(*probe.shape, *t.shape[nb:]), batch_size=probe.shape)

    def transpose(self, dim0: int, dim1: int) -> TensorDict:
        nb = len(self._batch_size)
        d0, d1 = dim0 % nb, dim1 % nb
        bs = list(self._batch_size)
        bs[d0], bs[d1] = bs[d1], bs[d0]
        return self.apply(lambda t: t.transpose(d0, d1), batch_size=bs)

    def permute(self, *dims: int) -> TensorDict:
        if len(dims) == 1 and isinstance(dims[0], (tuple, list)):
            dims = tuple(dims[0])
        nb = len(self._batch_size)
        bs = [self._batch_size[d] for d in dims]
        return self.apply(lambda t: t.permute(*dims, *range(nb, t.dim())), batch_size=bs)

    def unsqueeze(self, dim: int) -> TensorDict:
        nb = len(self._batch_size)
        d = dim if dim >= 0 else dim + nb + 1
        bs = list(self._batch_size)
        bs.insert(d, 1)
        return self.apply(lambda t: t.unsqueeze(d), batch_size=bs)

    def squeeze(self, dim: int) -> TensorDict:
        nb = len(self._batch_size)
        d = dim % nb
        bs = list(self._batch_size)
        if bs[d] != 1:
            return self
        bs.pop(d)
        return self.apply(lambda t: t.squeeze(d), batch_size=bs)

    def repeat(self, *sizes: int) -> TensorDict:
        nb = len(self._batch_size)
        bs = [b * s for b, s in zip(self._batch_size, sizes)]
        return self.apply(lambda t: t.repeat(*sizes, *([1] * (t.dim() - nb))), batch_size=bs)

    def split(self, split_size: int | list[int], dim: int = 0) -> tuple[TensorDict, ...]:
        parts = {k: v.split(split_size, dim) for k, v in self._data.items()}
        n = len(next(iter(parts.values()))) if parts else 0
        out = []
        for i in range(n):
            data = {k: p[i] for k, p in parts.items()}
            bs = list(self._batch_size)
            bs[dim] = next(iter(data.values())).shape[dim]
            out.append(TensorDict._from_parts(data, torch.Size(bs), self._device))
        return tuple(out)

    def __repr__(self) -> str:
        fields = ", ".join(f"{k}: {tuple(v.shape)} {v.dtype}" for k, v in self._data.items())
        return f"TensorDict({{{fields}}}, batch_size={tuple(self._batch_size)}, device={self.device})"

    def __eq__(self, other: object) -> Any:  # elementwise like tensordict
        if not isinstance(other, (TensorDict, Mapping)):
            return NotImplemented
        return TensorDict._from_parts({k: v == other[k] for k, v in self._data.items()}, self._batch_size,
                                      self._device)

    def all(self) -> bool:
        return all(bool(v.all()) for v in self._data.values())

    # ---- torch function protocol ----------------------------------------------------------------------------------
    @classmethod
    def __torch_function__(cls, func: Callable, types: Any, args: tuple = (), kwargs: dict | None = None) -> Any:
        kwargs = kwargs or {}
        if func in _TORCH_FUNCTIONS:
            return _TORCH_FUNCTIONS[func](*args, **kwargs)
        return NotImplemented


@_implements(torch.cat)
def _cat(tds: list[TensorDict] | tuple[TensorDict, ...], dim: int = 0, **_: Any) -> TensorDict:
    first = tds[0]
    nb = len(first.batch_size)
    d = dim % nb
    data = {k: torch.cat([td[k] for td in tds], dim=d) for k in first.keys()}
    bs = list(first.batch_size)
    bs[d] = sum(td.batch_size[d] for td in tds)
    return TensorDict._from_parts(data, torch.Size(bs), first._device)


@_implements(torch.stack)
def _stack(tds: list[TensorDict] | tuple[TensorDict, ...], dim: int = 0, **_: Any) -> TensorDict:
    first = tds[0]
    data = {k: torch.stack([td[k] for td in tds], dim=dim) for k in first.keys()}
    bs = list(first.batch_size)
    bs.insert(dim, len(tds))
    return TensorDict._from_parts(data, torch.Size(bs), first._device)


def is_tensordict(obj: Any) -> bool:
    """True for this class and for ``tensordict.TensorDict`` instances."""
    if isinstance(obj, TensorDict):
        return True
    return type(obj).__name__ == "TensorDict" and hasattr(obj, "batch_size")
