"""ctypes binding of the C ABI declared in ``include/w8a8_tp.h``.

The shared library ``_w8a8_tp.so`` is built in-tree by ``build.py``.  There is
no fallback: if the library is missing, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_w8a8_tp.so")

# Status codes (enum w8a8_status).
OK = 0
ERR_INVALID_ARG = 1
ERR_ALIGNMENT = 2
ERR_CUDA = 3
ERR_UNSUPPORTED = 4
ERR_TIMEOUT = 5
ERR_WORKSPACE = 6
ERR_STATE = 7

_STATUS_NAMES = {
    OK: "OK", ERR_INVALID_ARG: "INVALID_ARG", ERR_ALIGNMENT: "ALIGNMENT", ERR_CUDA: "CUDA",
    ERR_UNSUPPORTED: "UNSUPPORTED", ERR_TIMEOUT: "TIMEOUT", ERR_WORKSPACE: "WORKSPACE",
    ERR_STATE: "STATE",
}


class W8A8Error(RuntimeError):
    """Raised when a C-ABI call returns a non-zero status (mirrors PanicError)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{_STATUS_NAMES.get(status, status)}] {message}")
        self.status = status


_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size = ctypes.c_size_t

# name -> (restype, argtypes); the exact list of symbols include/w8a8_tp.h declares
SIGNATURES = {
    "w8a8_last_error": (ctypes.c_char_p, []),
    "w8a8_abi_version": (_c_int, []),
    "w8a8_device_error": (_c_int, [ctypes.POINTER(_c_int), _c_int]),
    "w8a8_quant_per_token": (_c_int, [_c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "w8a8_silu_mul_quant": (_c_int, [_c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "w8a8_quant_rows_amax": (_c_int, [_c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "w8a8_rmsnorm_quant": (_c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_vp, ctypes.c_float, _c_vp, _c_vp,
                                    _c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "w8a8_moe_max_blocks": (_c_i64, [_c_i64, _c_i64]),
    "w8a8_moe_align": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp]),
    "w8a8_moe_quant_scatter": (_c_int, [_c_vp, _c_i64, _c_i64, _c_i64, _c_vp, _c_int, _c_vp, _c_vp, _c_vp]),
    "w8a8_moe_gemm": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_vp,
                               _c_vp, _c_int, _c_i64, _c_i64, _c_vp]),
    "w8a8_moe_quant_rows": (_c_int, [_c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp]),
    "w8a8_moe_sum": (_c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_int, _c_i64, _c_vp, _c_i64, _c_vp]),
    "w8a8_gemm_workspace_size": (_c_size, [_c_i64, _c_i64, _c_i64]),
    "w8a8_gemm": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                           _c_i64, _c_i64, _c_i64, _c_vp, _c_size, _c_vp]),
    "w8a8_gemm_silu": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                                _c_i64, _c_i64, _c_i64, _c_vp, _c_size, _c_vp]),
    "w8a8_gemm_config": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                                  _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_vp, _c_size, _c_vp]),
    "w8a8_gemm_static_scratch": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                                          _c_i64, _c_i64, _c_i64, _c_vp]),
    "w8a8_mma_peak_probe": (_c_int, [_c_int, _c_i64, ctypes.POINTER(_c_i64), _c_vp]),
    "w8a8_gemm_plan": (_c_int, [_c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_size, _c_int,
                                ctypes.POINTER(_c_i64)]),
    "w8a8_comm_handle_bytes": (_c_size, []),
    "w8a8_comm_create": (_c_int, [_c_int, _c_int, _c_int, _c_size, ctypes.POINTER(_c_vp), _c_vp]),
    "w8a8_comm_open_peers": (_c_int, [_c_vp, _c_vp]),
    "w8a8_comm_set_mode": (_c_int, [_c_vp, _c_int]),
    "w8a8_comm_attach_multicast": (_c_int, [_c_vp, _c_vp, _c_vp, _c_size]),
    "w8a8_comm_set_timeout_ms": (_c_int, [_c_vp, _c_i64]),
    "w8a8_all_reduce": (_c_int, [_c_vp, _c_vp, _c_i64, _c_vp]),
    "w8a8_broadcast": (_c_int, [_c_vp, _c_vp, _c_i64, _c_int, _c_vp]),
    "w8a8_gemm_allreduce": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
                                     _c_i64, _c_i64, _c_i64, _c_vp, _c_size, _c_vp]),
    "w8a8_comm_status": (_c_int, [_c_vp, ctypes.POINTER(_c_int)]),
    "w8a8_comm_destroy": (None, [_c_vp]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load (once) the in-tree library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise W8A8Error(ERR_UNSUPPORTED,
                                f"{LIB_PATH} is not built; run `python mini-sglang-fork_b200/build.py`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().w8a8_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    if status != OK:
        msg = last_error()
        raise W8A8Error(status, f"{what}: {msg}" if what else msg)
