"""NVLink peer-memory communicator for the row-parallel all-reduce.

Counterpart of mini-sglang's ``init_pynccl`` / ``NCCLWrapper``
(M/kernel/pynccl.py:45-78, M/kernel/csrc/src/pynccl.cu:74-134): every rank
creates its IPC-shared buffer through the C ABI, the opaque handle blobs are
all-gathered over the CPU process group (as the NCCL unique id is broadcast
there), and every rank maps its peers' buffers.  ``all_reduce`` is the
in-place sum; ``gemm_allreduce`` is the row-parallel W8A8 linear with the
reduction fused into the GEMM kernel.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib, ops

__all__ = ["PeerMemCommunicator", "exchange_handles"]


def exchange_handles(blob: bytes, world: int, group=None) -> bytes:
    """All-gather every rank's handle blob in rank order over ``group``."""
    import torch.distributed as dist

    gathered = [None] * world
    dist.all_gather_object(gathered, blob, group=group)
    if any(g is None or len(g) != len(blob) for g in gathered):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "peer handle exchange returned malformed blobs")
    return b"".join(gathered)


class PeerMemCommunicator:
    """One rank's end of the peer-memory communicator.

    ``max_bytes`` bounds the bf16 tensor an ``all_reduce`` / ``gemm_allreduce``
    may produce (the reference sizes its symmetric buffer the same way,
    max_forward_len * hidden * itemsize, M/engine/engine.py:123-126).
    """

    def __init__(self, rank: int, world: int, max_bytes: int, cpu_group=None,
                 device: Optional[torch.device] = None, lib=None, timeout_ms: Optional[int] = None,
                 nvls: bool = True, device_group=None):
        self.rank = rank
        self.world = world
        self.max_bytes = int(max_bytes)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._lib = lib if lib is not None else _lib.load()
        self._handle = ctypes.c_void_p()
        nbytes = int(self._lib.w8a8_comm_handle_bytes())
        blob = ctypes.create_string_buffer(nbytes)
        dev_index = self.device.index if self.device.index is not None else 0
        _lib_check(self._lib, self._lib.w8a8_comm_create(rank, world, dev_index, self.max_bytes,
                                                         ctypes.byref(self._handle), blob), "comm_create")
        try:
            all_blobs = exchange_handles(blob.raw, world, cpu_group) if world > 1 else blob.raw
            buf = ctypes.create_string_buffer(all_blobs, len(all_blobs))
            _lib_check(self._lib, self._lib.w8a8_comm_open_peers(self._handle, buf), "comm_open_peers")
            if timeout_ms is not None:
                _lib_check(self._lib, self._lib.w8a8_comm_set_timeout_ms(self._handle, int(timeout_ms)),
                           "comm_set_timeout_ms")
        except BaseException:
            self.close()
            raise
        self.nvls_error: Optional[str] = None
        self._nv_buf = self._nv_handle = None
        if world > 1 and nvls:
            self._attach_multicast(device_group)

    def _attach_multicast(self, group) -> None:
        """NVSwitch multicast buffer for the fused reduce (4 x max_bytes: two
        halves of [partials | gathered shares]), allocated and mapped by
        torch's symmetric memory -- plumbing only; the multimem loads and
        stores are this package's kernels.  Collective over ``group`` (the
        default group when None).  Without multicast support the fused reduce
        keeps its peer-store two-shot; the reason is kept in ``nvls_error``."""
        try:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm

            nbytes = 4 * ((self.max_bytes + 4095) // 4096 * 4096)
            buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
            handle = symm.rendezvous(buf, group if group is not None else dist.group.WORLD)
            mc = int(handle.multicast_ptr)
            if not mc:
                raise RuntimeError("no multicast mapping (NVLS unsupported here)")
            uc = int(handle.buffer_ptrs[self.rank])
            # the multicast address maps this allocation from its base: use it only
            # for a handle that starts there and covers the whole buffer
            if int(handle.offset) != 0 or uc != buf.data_ptr() or int(handle.buffer_size) < nbytes:
                raise RuntimeError("symmetric buffer is not a whole allocation of its own")
            _lib_check(self._lib, self._lib.w8a8_comm_attach_multicast(self._handle, mc, uc, nbytes),
                       "comm_attach_multicast")
            self._nv_buf, self._nv_handle = buf, handle
        except Exception as e:  # noqa: BLE001 - reported through nvls_error
            self.nvls_error = f"{type(e).__name__}: {e}"[:300]

    @property
    def nvls(self) -> bool:
        """True once a multicast buffer is attached (NVLS fused reduce available)."""
        return self._nv_buf is not None

    def set_mode(self, mode: int) -> None:
        """Algorithm: 0 automatic, 1 one-shot, 2 two-shot (peer stores), 3 the
        fused GEMM's two-shot through NVLS (needs the multicast buffer)."""
        _lib_check(self._lib, self._lib.w8a8_comm_set_mode(self._handle, int(mode)), "comm_set_mode")

    # -------------------------------------------------------------- collectives
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        """In-place sum over the ranks (fp32 rank-order sum, one bf16 rounding)."""
        if (x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous()
                or x.device.index != self.device.index):
            raise _lib.W8A8Error(_lib.ERR_INVALID_ARG,
                                 "all_reduce: contiguous bf16 tensor on the communicator's device required")
        st = self._lib.w8a8_all_reduce(self._handle, x.data_ptr(), x.numel(),
                                       torch.cuda.current_stream(x.device).cuda_stream)
        _lib_check(self._lib, st, "all_reduce")
        return x

    def broadcast(self, x: torch.Tensor, root: int = 0) -> torch.Tensor:
        """In-place broadcast of ``x`` from rank ``root`` (every rank passes a
        tensor of the same size; the others' contents are overwritten)."""
        if not x.is_cuda or not x.is_contiguous() or x.device.index != self.device.index:
            raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "broadcast: contiguous tensor on the communicator's device required")
        st = self._lib.w8a8_broadcast(self._handle, x.data_ptr(), x.numel() * x.element_size(), int(root),
                                      torch.cuda.current_stream(x.device).cuda_stream)
        _lib_check(self._lib, st, "broadcast")
        return x

    def gemm_allreduce(self, aq: torch.Tensor, wq: torch.Tensor, sa: torch.Tensor, sw: torch.Tensor,
                       bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Row-parallel W8A8 linear of this rank's K-shard, all-reduced over the
        ranks inside the GEMM kernel; every rank returns the full sum."""
        m, n, k, out = ops.check_gemm_operands("gemm_allreduce", aq, wq, sa, sw, bias, out)
        if aq.device.index != self.device.index:
            raise _lib.W8A8Error(_lib.ERR_INVALID_ARG,
                                 f"gemm_allreduce: operands on {aq.device}, communicator on {self.device}")
        ws = ops.gemm_workspace(aq.device)
        st = self._lib.w8a8_gemm_allreduce(self._handle, aq.data_ptr(), wq.data_ptr(), sa.data_ptr(),
                                           sw.data_ptr(), None if bias is None else bias.data_ptr(),
                                           out.data_ptr(), m, n, k, ws.data_ptr(), ws.numel(),
                                           torch.cuda.current_stream(aq.device).cuda_stream)
        _lib_check(self._lib, st, "gemm_allreduce")
        return out

    def device_error(self) -> int:
        """Non-zero once a bounded cross-rank wait gave up (synchronises)."""
        code = ctypes.c_int(0)
        _lib_check(self._lib, self._lib.w8a8_comm_status(self._handle, ctypes.byref(code)), "comm_status")
        return code.value

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            self._lib.w8a8_comm_destroy(self._handle)
            self._handle = ctypes.c_void_p()
        self._nv_buf = self._nv_handle = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


def _lib_check(lib, status: int, what: str) -> None:
    if status != _lib.OK:
        msg = lib.w8a8_last_error()
        msg = msg.decode(errors="replace") if isinstance(msg, bytes) else str(msg)
        raise _lib.W8A8Error(status, f"{what}: {msg}")
