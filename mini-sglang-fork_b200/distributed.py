"""Tensor-parallel geometry and the all-reduce plugin stack.

Inside mini-sglang the layers use the reference's own state: when
``minisgl.distributed`` (M/distributed/) is importable and its
``set_tp_info`` has been called, ``get_tp_info`` returns the reference's
``DistributedInfo``, ``communicator()`` returns the reference's
``DistributedCommunicator`` (so a row-parallel layer without the fused reduce
all-reduces through whatever plugin the engine enabled, PyNCCL included), and
``enable_peer_mem_distributed`` appends its plugin to the reference's plugin
list exactly as ``enable_pynccl_distributed`` does (M/distributed/impl.py:73-90).

Standalone (the reference not importable, or its TP info unset) the same
surface is served by this module's own copy of it, mirroring
M/distributed/info.py:1-38 and M/distributed/impl.py:15-97: a process-global
``DistributedInfo`` set once per rank and a ``DistributedCommunicator`` that
dispatches ``all_reduce`` / ``all_gather`` to the last registered plugin.
``TorchDistributedImpl`` is the plain ``torch.distributed`` plugin (NCCL on
GPUs, gloo on CPU ranks); ``PeerMemDistributedImpl`` routes ``all_reduce`` to
this package's NVLink peer-memory communicator.
"""
from __future__ import annotations

import importlib
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import TYPE_CHECKING, List, Optional

import torch
import torch.distributed as dist

if TYPE_CHECKING:
    from .comm import PeerMemCommunicator

__all__ = [
    "DistributedInfo",
    "set_tp_info",
    "get_tp_info",
    "try_get_tp_info",
    "reset_tp_info",
    "DistributedImpl",
    "TorchDistributedImpl",
    "PeerMemDistributedImpl",
    "DistributedCommunicator",
    "enable_peer_mem_distributed",
    "get_peer_mem_comm",
    "destroy_distributed",
    "div_even",
    "communicator",
    "reference_distributed",
]


def reference_distributed():
    """The reference's ``minisgl.distributed`` module when it is importable
    (mini-sglang installed beside this package), else None."""
    try:
        return importlib.import_module("minisgl.distributed")
    except ImportError:
        return None


def _bound_reference():
    """The reference's module when the layers should use its state: it is
    importable, its TP info is set and this module's own is not."""
    if _TP_INFO is not None:
        return None
    ref = reference_distributed()
    if ref is None or ref.try_get_tp_info() is None:
        return None
    return ref


@dataclass(frozen=True)
class DistributedInfo:
    """TP rank and size of this process (M/distributed/info.py:6-15)."""

    rank: int
    size: int

    def __post_init__(self):
        assert 0 <= self.rank < self.size

    def is_primary(self) -> bool:
        return self.rank == 0


_TP_INFO: Optional[DistributedInfo] = None


def set_tp_info(rank: int, size: int) -> None:
    """Set the process-global TP info once (M/distributed/info.py:21-25)."""
    global _TP_INFO
    if _TP_INFO is not None:
        raise RuntimeError("TP info has been set")
    _TP_INFO = DistributedInfo(rank, size)


def get_tp_info() -> DistributedInfo:
    """This process's TP info: this module's own when set, else the
    reference's (M/distributed/info.py:28-31) when it has been set there."""
    if _TP_INFO is not None:
        return _TP_INFO
    ref = _bound_reference()
    if ref is not None:
        return ref.get_tp_info()
    raise RuntimeError("TP info has not been set")


def try_get_tp_info() -> Optional[DistributedInfo]:
    if _TP_INFO is not None:
        return _TP_INFO
    ref = _bound_reference()
    return ref.try_get_tp_info() if ref is not None else None


def reset_tp_info() -> None:
    """Clear the TP info (test harnesses that emulate several ranks in one process)."""
    global _TP_INFO
    _TP_INFO = None


def div_even(a: int, b: int, allow_replicate: bool = False) -> int:
    """``a / b`` that must divide evenly; ``allow_replicate`` returns 1 when
    ``b > a`` and ``a`` divides ``b`` (KV-head replication), as
    M/utils/misc.py:20-26."""
    if allow_replicate and b > a:
        if b % a != 0:
            raise AssertionError(f"b = {b} must be divisible by a = {a} for KV head replication")
        return 1
    if a % b != 0:
        raise AssertionError(f"a = {a} must be divisible by b = {b}")
    return a // b


class DistributedImpl(ABC):
    @abstractmethod
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor: ...

    @abstractmethod
    def all_gather(self, x: torch.Tensor) -> torch.Tensor: ...


class TorchDistributedImpl(DistributedImpl):
    """``torch.distributed`` collectives on the default group (M/distributed/impl.py:24-41)."""

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if dist.get_world_size() == 1:
            return x
        dist.all_reduce(x, op=dist.ReduceOp.SUM)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size()
        if world == 1:
            return x
        shape = list(x.shape)
        shape[0] *= world
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x)
        return out


class PeerMemDistributedImpl(DistributedImpl):
    """``all_reduce`` through the NVLink peer-memory communicator (in place)."""

    def __init__(self, comm: "PeerMemCommunicator"):
        self.comm = comm

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        self.comm.all_reduce(x)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return TorchDistributedImpl().all_gather(x)


class DistributedCommunicator:
    """Dispatch to the last registered plugin (M/distributed/impl.py:63-70)."""

    plugins: List[DistributedImpl] = [TorchDistributedImpl()]

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_gather(x)


def communicator():
    """The all-reduce dispatcher the row-parallel layers fall back to when
    the reduce is not fused: the reference's ``DistributedCommunicator`` when
    its state is in use (so the engine's PyNCCL plugin is reached), else this
    module's."""
    ref = _bound_reference()
    return ref.DistributedCommunicator() if ref is not None else DistributedCommunicator()


_PEER_MEM_COMM: Optional["PeerMemCommunicator"] = None


def enable_peer_mem_distributed(tp_info: DistributedInfo, tp_cpu_group, max_bytes: int,
                                device: Optional[torch.device] = None,
                                device_group=None) -> Optional["PeerMemCommunicator"]:
    """Create the peer-memory communicator and register it as the all-reduce
    plugin; the W8A8 row-parallel layers then fuse their reduction into the
    GEMM.  Counterpart of ``enable_pynccl_distributed`` (M/distributed/impl.py:73-90):
    handles are exchanged over ``tp_cpu_group`` as the NCCL unique id is; the
    NVSwitch multicast buffer (when the machine has NVLS) is set up over
    ``device_group`` (the default group when None)."""
    global _PEER_MEM_COMM
    if tp_info.size == 1:
        return None
    from .comm import PeerMemCommunicator

    comm = PeerMemCommunicator(tp_info.rank, tp_info.size, max_bytes, tp_cpu_group, device=device,
                               device_group=device_group)
    _PEER_MEM_COMM = comm
    plugin = PeerMemDistributedImpl(comm)
    DistributedCommunicator.plugins.append(plugin)
    ref = _bound_reference()
    if ref is not None:  # the engine's own dispatcher reaches it too, as PyNCCL's plugin does
        ref.DistributedCommunicator.plugins.append(plugin)
    return comm


def get_peer_mem_comm() -> Optional["PeerMemCommunicator"]:
    return _PEER_MEM_COMM


def destroy_distributed() -> None:
    """Drop every plugin and the peer-memory communicator (M/distributed/impl.py:93-97);
    this package's plugin also leaves the reference's list."""
    global _PEER_MEM_COMM
    ref = reference_distributed()
    if ref is not None:
        ref.DistributedCommunicator.plugins = [p for p in ref.DistributedCommunicator.plugins
                                               if not isinstance(p, PeerMemDistributedImpl)]
    if _PEER_MEM_COMM is not None:
        _PEER_MEM_COMM.close()
    _PEER_MEM_COMM = None
    DistributedCommunicator.plugins = []
