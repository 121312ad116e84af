"""W8A8 tensor-parallel linear layers with mini-sglang's operator surface.

Same class names, constructor signatures, size bookkeeping and state-dict
rules as mini-sglang's bf16 layers (M/layers/linear.py:13-127,
M/layers/base.py:15-99); the weight is held as int8 ``weight [N_local,
K_local]`` plus ``weight_scale [N_local]`` fp32, and ``forward`` runs the
per-token quantiser and the tcgen05 int8 GEMM.  Row-parallel layers return
the all-reduced output like the reference; when a peer-memory communicator is
enabled the reduction is fused into the GEMM, otherwise the plugin stack's
``all_reduce`` runs after it.

Weight sharding (for loaders): quantise the UNSHARDED bf16 weight per output
channel, then shard ``weight`` exactly like the bf16 tensor
(M/models/weight.py:34-52); ``weight_scale`` follows dim-0 shards
(column-parallel) and is replicated for dim-1 shards (row-parallel).
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Union

import torch

from . import ops
from .distributed import communicator, div_even, get_peer_mem_comm, get_tp_info
from .ops import QuantizedActivation

_STATE_DICT = Dict[str, torch.Tensor]

__all__ = [
    "BaseOP",
    "LinearReplicated",
    "LinearColParallelMerged",
    "LinearQKVMerged",
    "LinearOProj",
    "LinearRowParallel",
    "GatedMLP",
    "MoELayer",
    "silu_and_mul",
    "silu_and_mul_quant",
]

silu_and_mul = ops.silu_and_mul
silu_and_mul_quant = ops.silu_and_mul_quant


def _concat_prefix(prefix: str, name: str) -> str:
    return f"{prefix}.{name}" if prefix else name


class BaseOP:
    """State-dict discovery of every public tensor / sub-op attribute, as
    ``BaseOP`` does (M/layers/base.py:15-53): names starting with ``_`` are
    private; ``load_state_dict`` replaces each tensor after checking that shape
    and dtype match."""

    def forward(self, *args: Any, **kwargs: Any) -> Any:  # pragma: no cover - abstract
        raise NotImplementedError

    def state_dict(self, *, prefix: str = "", result: Optional[_STATE_DICT] = None) -> _STATE_DICT:
        result = result if result is not None else {}
        for name, value in self.__dict__.items():
            if name.startswith("_"):
                continue
            if isinstance(value, torch.Tensor):
                result[_concat_prefix(prefix, name)] = value
            elif isinstance(value, BaseOP):
                value.state_dict(prefix=_concat_prefix(prefix, name), result=result)
        return result

    def load_state_dict(self, state_dict: _STATE_DICT, *, prefix: str = "", _internal: bool = False) -> None:
        for name, value in list(self.__dict__.items()):
            if name.startswith("_"):
                continue
            if isinstance(value, torch.Tensor):
                item = state_dict.pop(_concat_prefix(prefix, name))
                if not isinstance(item, torch.Tensor):
                    raise TypeError(f"{_concat_prefix(prefix, name)} is not a tensor")
                if value.shape != item.shape or value.dtype != item.dtype:
                    raise ValueError(f"{_concat_prefix(prefix, name)}: expected {tuple(value.shape)} {value.dtype}, "
                                     f"got {tuple(item.shape)} {item.dtype}")
                setattr(self, name, item)
            elif isinstance(value, BaseOP):
                value.load_state_dict(state_dict, prefix=_concat_prefix(prefix, name), _internal=True)
        if not _internal and state_dict:
            raise RuntimeError(f"Unexpected keys in state_dict: {list(state_dict.keys())}")


class _LinearTPImpl(BaseOP):
    """W8A8 counterpart of ``_LinearTPImpl`` (M/layers/linear.py:13-32)."""

    def __init__(self, full_isize: int, full_osize: int, local_isize: int, local_osize: int, has_bias: bool):
        self.full_input_size = full_isize
        self.full_output_size = full_osize
        self.local_input_size = local_isize
        self.local_output_size = local_osize
        self.weight = torch.empty(local_osize, local_isize, dtype=torch.int8)
        self.weight_scale = torch.empty(local_osize, dtype=torch.float32)
        self.bias = torch.empty(local_osize, dtype=torch.bfloat16) if has_bias else None

    def _quantize_input(self, x: Union[torch.Tensor, QuantizedActivation]) -> QuantizedActivation:
        if isinstance(x, QuantizedActivation):
            return x
        q, s = ops.quant_per_token(x)
        return QuantizedActivation(q, s)

    def forward(self, x: Union[torch.Tensor, QuantizedActivation]) -> torch.Tensor:
        qa = self._quantize_input(x)
        return ops.w8a8_gemm(qa.q, self.weight, qa.s, self.weight_scale, self.bias)


class LinearReplicated(_LinearTPImpl):
    """Unsharded W8A8 linear (M/layers/linear.py:35-53)."""

    def __init__(self, input_size: int, output_size: int, has_bias: bool):
        super().__init__(input_size, output_size, input_size, output_size, has_bias)


class LinearColParallelMerged(_LinearTPImpl):
    """Column-parallel merged linear, e.g. gate_up (M/layers/linear.py:56-68)."""

    def __init__(self, input_size: int, output_sizes: List[int], has_bias: bool):
        tp_info = get_tp_info()
        tp_output_sizes = [div_even(size, tp_info.size) for size in output_sizes]
        super().__init__(input_size, sum(output_sizes), input_size, sum(tp_output_sizes), has_bias)

    def forward_silu_quant(self, x: Union[torch.Tensor, QuantizedActivation]) -> QuantizedActivation:
        """For a [gate; up] merge (GatedMLP's gate_up_proj): the quantised
        ``silu(gate) * up`` that ``silu_and_mul_quant(self.forward(x))`` gives,
        bit for bit, with the SiLU*mul in the GEMM's epilogue when the shape
        allows (ops.gate_up_silu_quant) so the [M, 2I] output is never
        written; otherwise in those two steps."""
        qa = self._quantize_input(x)
        fused = ops.gate_up_silu_quant(qa.q, self.weight, qa.s, self.weight_scale, self.bias)
        if fused is not None:
            return fused
        return ops.silu_and_mul_quant(ops.w8a8_gemm(qa.q, self.weight, qa.s, self.weight_scale, self.bias))


class LinearQKVMerged(_LinearTPImpl):
    """Column-parallel q|k|v over heads, kv replicated when kv_heads < tp
    (M/layers/linear.py:71-88)."""

    def __init__(self, hidden_size: int, head_dim: int, num_qo_heads: int, num_kv_heads: int, has_bias: bool):
        tp_info = get_tp_info()
        local_num_qo = div_even(num_qo_heads, tp_info.size)
        local_num_kv = div_even(num_kv_heads, tp_info.size, allow_replicate=True)
        full_osize = (num_qo_heads + 2 * num_kv_heads) * head_dim
        local_osize = (local_num_qo + 2 * local_num_kv) * head_dim
        super().__init__(hidden_size, full_osize, hidden_size, local_osize, has_bias)


class _RowParallel(_LinearTPImpl):
    """Row-parallel forward: local W8A8 GEMM of the K-shard, then the sum over
    ranks (M/layers/linear.py:102-106,123-127).  With a peer-memory
    communicator the reduction runs inside the GEMM kernel."""

    _tp_size: int
    _comm: object  # a DistributedCommunicator: the reference's when its state is in use

    def forward(self, x: Union[torch.Tensor, QuantizedActivation]) -> torch.Tensor:
        qa = self._quantize_input(x)
        if self._tp_size > 1:
            fused = get_peer_mem_comm()
            if fused is not None:
                return fused.gemm_allreduce(qa.q, self.weight, qa.s, self.weight_scale, self.bias)
            y = ops.w8a8_gemm(qa.q, self.weight, qa.s, self.weight_scale, self.bias)
            return self._comm.all_reduce(y)
        return ops.w8a8_gemm(qa.q, self.weight, qa.s, self.weight_scale, self.bias)


class LinearOProj(_RowParallel):
    """o_proj (M/layers/linear.py:91-106)."""

    def __init__(self, input_size: int, output_size: int, has_bias: bool):
        tp_info = get_tp_info()
        self._comm = communicator()
        self._tp_size = tp_info.size
        super().__init__(input_size, output_size, div_even(input_size, tp_info.size), output_size, has_bias)


class LinearRowParallel(_RowParallel):
    """down_proj (M/layers/linear.py:109-127)."""

    def __init__(self, input_size: int, output_size: int, has_bias: bool):
        tp_info = get_tp_info()
        self._comm = communicator()
        self._tp_size = tp_info.size
        super().__init__(input_size, output_size, div_even(input_size, tp_info.size), output_size, has_bias)


class RMSNormFusedQuant(BaseOP):
    """``RMSNormFused`` (M/layers/norm.py:23-38) with the following W8A8
    layer's input quantisation fused in: ``forward(x, residual)`` returns
    ``(QuantizedActivation, residual)`` -- the residual updated in place to
    ``x + residual`` as ``fused_add_rmsnorm`` does, or ``x`` itself without
    one -- and the bf16 normalised rows never reach HBM.  qkv / gate_up accept
    the QuantizedActivation directly.  ``weight`` is the bf16 [size] norm
    weight (state dict key ``weight``)."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size, dtype=torch.bfloat16)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None):
        return ops.rmsnorm_quant(x, self.weight, self.eps, residual)


class GatedMLP(BaseOP):
    """W8A8 ``GatedMLP`` (M/models/utils.py:25-50): gate_up (column-parallel)
    with SiLU*mul in its epilogue -> per-token quant -> down (row-parallel +
    all-reduce).  The [M, 2I] gate_up output never touches HBM (below the
    fusion's shape range: gate_up, then the fused SiLU*mul quantiser)."""

    def __init__(self, hidden_size: int, intermediate_size: int):
        self.gate_up_proj = LinearColParallelMerged(hidden_size, [intermediate_size, intermediate_size],
                                                    has_bias=False)
        self.down_proj = LinearRowParallel(intermediate_size, hidden_size, has_bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.gate_up_proj.forward_silu_quant(x)
        del x
        return self.down_proj.forward(y)


class MoELayer(BaseOP):
    """W8A8 ``MoELayer`` (M/layers/moe.py:8-58): the experts of a mixture-of-
    experts MLP, TP-sharded on the intermediate dim like the reference's
    (``intermediate_size / tp`` per rank).  State dict: ``gate_up_proj`` int8
    [E, 2I_local, H] ([gate; up] per expert), ``gate_up_proj_scale`` fp32
    [E, 2I_local], ``down_proj`` int8 [E, H, I_local], ``down_proj_scale``
    fp32 [E, H] (per output channel of the unsharded weights, replicated on
    the dim-1 shards as for the dense layers).  ``forward(hidden_states,
    router_logits)`` routes with the reference's ``fused_topk`` arithmetic
    (softmax in fp32, top-k, optional renormalisation; torch ops on the
    device), runs :func:`ops.fused_experts_w8a8` and, for tp > 1, the
    plugin stack's ``all_reduce``.  Only ``activation="silu"`` with the
    routing weight on the down projection (the reference's defaults) exists
    in W8A8."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 renormalize: bool = True, activation: str = "silu",
                 apply_router_weight_on_input: bool = False):
        if activation != "silu" or apply_router_weight_on_input:
            raise ValueError("MoELayer (W8A8): only activation='silu' with the routing weight on the down "
                             "projection is provided")
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.renormalize = renormalize
        self.activation = activation
        self.apply_router_weight_on_input = apply_router_weight_on_input
        self._comm = communicator()
        self.tp_size = tp_size = get_tp_info().size
        i_local = div_even(intermediate_size, tp_size)
        self.gate_up_proj = torch.empty(num_experts, 2 * i_local, hidden_size, dtype=torch.int8)
        self.gate_up_proj_scale = torch.empty(num_experts, 2 * i_local, dtype=torch.float32)
        self.down_proj = torch.empty(num_experts, hidden_size, i_local, dtype=torch.int8)
        self.down_proj_scale = torch.empty(num_experts, hidden_size, dtype=torch.float32)

    def route(self, router_logits: torch.Tensor):
        """``fused_topk`` (M/moe/fused.py:9-29): ``(topk_weights fp32, topk_ids
        int32)``, both [T, top_k]."""
        p = torch.softmax(router_logits.float(), dim=-1)
        w, ids = torch.topk(p, self.top_k, dim=-1)
        if self.renormalize:
            w = w / w.sum(dim=-1, keepdim=True)
            w = w / (w.sum(dim=-1, keepdim=True) + 1e-8)
        return w.contiguous(), ids.to(torch.int32).contiguous()

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        topk_weights, topk_ids = self.route(router_logits)
        out = ops.fused_experts_w8a8(hidden_states, self.gate_up_proj, self.gate_up_proj_scale, self.down_proj,
                                     self.down_proj_scale, topk_weights, topk_ids)
        if self.tp_size > 1:
            out = self._comm.all_reduce(out)
        return out
