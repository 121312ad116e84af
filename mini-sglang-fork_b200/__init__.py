"""B200-native W8A8 tensor-parallel linear path for mini-sglang's model code.

Hand-written sm_100a CUDA (``csrc/``) behind a C ABI (``include/w8a8_tp.h``),
bound with ctypes (``_lib``), wrapped for torch tensors (``ops``) and exposed
through mini-sglang's layer surface (``layers``, ``distributed``, ``comm``).

The directory name is not a Python identifier; import it with
``importlib.import_module("mini-sglang-fork_b200")`` (repository root on
``sys.path``).
"""
from __future__ import annotations

from . import _lib, comm, distributed, layers, ops, weights
from ._lib import W8A8Error
from .distributed import (DistributedCommunicator, DistributedInfo, destroy_distributed,
                          enable_peer_mem_distributed, get_tp_info, reset_tp_info, set_tp_info,
                          try_get_tp_info)
from .layers import (BaseOP, GatedMLP, LinearColParallelMerged, LinearOProj, LinearQKVMerged,
                     LinearReplicated, LinearRowParallel, MoELayer, RMSNormFusedQuant, silu_and_mul,
                     silu_and_mul_quant)
from .ops import QuantizedActivation, quant_per_token, w8a8_gemm
from .weights import load_w8a8_state_dict, w8a8_weight_stream

__all__ = [
    "W8A8Error",
    "BaseOP",
    "GatedMLP",
    "MoELayer",
    "LinearColParallelMerged",
    "LinearOProj",
    "LinearQKVMerged",
    "LinearReplicated",
    "LinearRowParallel",
    "RMSNormFusedQuant",
    "QuantizedActivation",
    "quant_per_token",
    "silu_and_mul",
    "silu_and_mul_quant",
    "w8a8_gemm",
    "load_w8a8_state_dict",
    "w8a8_weight_stream",
    "DistributedCommunicator",
    "DistributedInfo",
    "set_tp_info",
    "get_tp_info",
    "try_get_tp_info",
    "reset_tp_info",
    "enable_peer_mem_distributed",
    "destroy_distributed",
    "load_library",
]


def load_library():
    """Load the in-tree CUDA library (raises if it is not built)."""
    return _lib.load()
