"""W8A8 checkpoint loading: the int8 counterpart of mini-sglang's streaming
weight loader (M/models/weight.py), producing the state dict the W8A8 layer
classes of ``layers.py`` expect.

It consumes (name, tensor) pairs -- what ``safetensors.safe_open(...).keys()``
/ ``get_tensor`` yield in the reference's ``load_weight`` (weight.py:76-125) --
and yields this rank's (name, tensor) pairs, sharded and merged:

* sharding is positional, exactly as ``_shard_tensor`` (weight.py:34-52):
  q/k/v/gate/up split on dim 0 (k/v by whole heads, replicated when the kv
  heads are fewer than the ranks), o/down split on dim 1, lm_head /
  embed_tokens split by vocabulary rows, everything else unsharded;
* merge groups follow ``_MERGE_GROUPS`` (weight.py:13-30): q|k|v ->
  qkv_proj and gate|up -> gate_up_proj, concatenated on dim 0 in slot order;
* ``<proj>.weight_scale`` (fp32 [N], one per output channel) follows its
  weight's rows on dim-0 splits and is replicated on dim-1 splits (every rank
  needs the scale of every output channel), and is merged like the weight;
* an int8 checkpoint (``.weight`` int8 + ``.weight_scale``) is passed through
  that rule as is; a bf16 / fp16 / fp32 checkpoint is quantised at load time,
  per output channel on the UNSHARDED weight (s = amax/127, round half even),
  then sharded -- so every rank's shard carries the same scales the unsharded
  weight had.

Quantisation at load runs the library's CUDA quantiser on the weight rows
(``ops.quant_per_token``: per-row absmax == per-output-channel for a
[N, K] weight) on ``device``; there is no CPU quantiser in the product.
* MoE experts (``num_experts`` given): every ``<prefix>.experts.<i>.<name>``
  tensor, once sharded and merged, is held until all experts have it and then
  yielded stacked on a new dim 0 under ``<prefix>.<name>`` with ``.weight``
  dropped -- the reference's ``_get_expert_stack_info`` / ``torch.stack``
  (weight.py:62-73,111-119); the scale ``...gate_up_proj.weight_scale``
  stacks under ``...gate_up_proj_scale``, the name ``MoELayer`` gives it.
"""
from __future__ import annotations

import re
from typing import Callable, Dict, Iterable, Iterator, Optional, Tuple

import torch

from . import _lib, ops

_SPLIT_DIM_0 = (".q_proj", ".k_proj", ".v_proj", ".gate_proj", ".up_proj")
_SPLIT_DIM_1 = (".o_proj", ".down_proj")
_KV = (".k_proj", ".v_proj")
# projection suffix -> (merged suffix, slot, slots in concatenation order)
_MERGE_GROUPS = {
    ".q_proj": (".qkv_proj", "q", ("q", "k", "v")),
    ".k_proj": (".qkv_proj", "k", ("q", "k", "v")),
    ".v_proj": (".qkv_proj", "v", ("q", "k", "v")),
    ".gate_proj": (".gate_up_proj", "gate", ("gate", "up")),
    ".up_proj": (".gate_up_proj", "up", ("gate", "up")),
}
_SKIP_PREFIXES = ("vision_tower.", "multi_modal_projector.")
_EXPERT = re.compile(r"^(?P<prefix>.+\.experts)\.(?P<idx>\d+)\.(?P<name>.+)$")

Quantiser = Callable[[torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]


def _div_ceil(a: int, b: int) -> int:
    return (a + b - 1) // b


def shard_tensor(key: str, value: torch.Tensor, rank: int, world: int,
                 num_kv_heads: Optional[int]) -> torch.Tensor:
    """This rank's shard of one checkpoint tensor: the positional split of
    ``_shard_tensor`` (M/models/weight.py:34-52).  Works for int8 weights as
    for bf16 ones, and for 1-D biases of dim-0 split projections."""
    if any(s in key for s in _SPLIT_DIM_0):
        if any(s in key for s in _KV) and num_kv_heads is not None and num_kv_heads < world:
            head_dim = value.shape[0] // num_kv_heads
            head = rank * num_kv_heads // world
            return value[head * head_dim:(head + 1) * head_dim].clone()
        return value.chunk(world, dim=0)[rank].clone()
    if any(s in key for s in _SPLIT_DIM_1):
        return value.chunk(world, dim=1)[rank].clone()
    if "lm_head" in key or "embed_tokens" in key:
        per_rank = _div_ceil(value.shape[0], world)
        return value[rank * per_rank:min((rank + 1) * per_rank, value.shape[0])].clone()
    return value


def shard_weight_scale(key: str, scale: torch.Tensor, rank: int, world: int,
                       num_kv_heads: Optional[int]) -> torch.Tensor:
    """This rank's per-output-channel scales: the weight's row split on dim-0
    splits, the whole vector on dim-1 (row-parallel) splits."""
    if scale.dim() != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{key}: weight_scale must be 1-D, got {tuple(scale.shape)}")
    if any(s in key for s in _SPLIT_DIM_1):
        return scale.clone()
    return shard_tensor(key, scale, rank, world, num_kv_heads)


def is_linear_weight(key: str) -> bool:
    """A weight of one of the W8A8 projections (q/k/v/o/gate/up/down), or the
    MoE router ``mlp.gate`` (a LinearReplicated in M/models/utils.py:62-66)."""
    return key.endswith(".weight") and (any(s in key for s in _SPLIT_DIM_0 + _SPLIT_DIM_1)
                                        or key.endswith(".mlp.gate.weight"))


def cuda_quantiser(device: torch.device) -> Quantiser:
    """Per-output-channel int8 quantisation of a [N, K] weight with the
    library's CUDA quantiser on ``device`` (raises without CUDA or the
    library, like every op)."""
    def quantise(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        if w.dim() != 2:
            raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"weight must be 2-D, got {tuple(w.shape)}")
        return ops.quant_per_token(w.to(device=device, dtype=torch.bfloat16).contiguous())
    return quantise


def _merge_info(key: str):
    for suffix, (fused, slot, slots) in _MERGE_GROUPS.items():
        if suffix in key:
            return key.replace(suffix, fused), slot, slots
    return None


def expert_stack_info(key: str) -> Optional[Tuple[str, int]]:
    """``(packed key, expert index)`` of an expert-scoped key, else None."""
    m = _EXPERT.match(key)
    if m is None:
        return None
    name = m.group("name")
    if name.endswith(".weight_scale"):
        name = name[: -len(".weight_scale")] + "_scale"
    elif name.endswith(".weight"):
        name = name[: -len(".weight")]
    return f"{m.group('prefix')}.{name}", int(m.group("idx"))


def _cast(key: str, value: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The engine's load-time cast to the model dtype (M/engine/engine.py:146),
    which must leave int8 weights and their fp32 scales alone."""
    if key.endswith(".weight_scale"):
        return value.to(torch.float32)
    if value.is_floating_point():
        return value.to(dtype)
    return value


def w8a8_weight_stream(items: Iterable[Tuple[str, torch.Tensor]], rank: int, world: int,
                       num_kv_heads: Optional[int], quantise: Optional[Quantiser] = None,
                       device: Optional[torch.device] = None,
                       dtype: torch.dtype = torch.bfloat16,
                       num_experts: Optional[int] = None) -> Iterator[Tuple[str, torch.Tensor]]:
    """Shard and merge a checkpoint stream for ``rank`` of ``world`` (see the
    module docstring).  ``quantise`` turns a floating [N, K] weight into
    (int8 [N, K], fp32 [N]); by default the CUDA quantiser on ``device``
    (the current CUDA device if None).  Floating tensors other than the scales
    (biases, norms, embeddings) are cast to ``dtype``.  Raises if a merge group
    is incomplete at the end of the stream; an int8 weight without its scale is
    caught by the layers' ``load_state_dict``.  With ``num_experts`` the
    experts' tensors are stacked (module docstring)."""
    if not (0 <= rank < world):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"rank {rank} not in [0, {world})")
    merge_buf: Dict[str, Dict[str, torch.Tensor]] = {}
    expert_buf: Dict[str, Dict[int, torch.Tensor]] = {}

    def out(key: str, value: torch.Tensor) -> Iterator[Tuple[str, torch.Tensor]]:
        info = expert_stack_info(key) if num_experts else None
        if info is None:
            yield key, value
            return
        packed, idx = info
        slots = expert_buf.setdefault(packed, {})
        slots[idx] = value
        if len(slots) == num_experts:
            del expert_buf[packed]
            yield packed, torch.stack([slots[i] for i in range(num_experts)], dim=0)

    for name, tensor in items:
        if name.startswith(_SKIP_PREFIXES):
            continue
        name = name.removeprefix("language_model.")
        if is_linear_weight(name) and tensor.is_floating_point():
            if quantise is None:  # created on first use: int8 checkpoints need no CUDA here
                quantise = cuda_quantiser(device if device is not None
                                          else torch.device("cuda", torch.cuda.current_device()))
            q, s = quantise(tensor)
            produced = [(name, shard_tensor(name, q, rank, world, num_kv_heads)),
                        (name + "_scale", shard_weight_scale(name, s, rank, world, num_kv_heads))]
        elif name.endswith(".weight_scale"):
            produced = [(name, shard_weight_scale(name, tensor.float(), rank, world, num_kv_heads))]
        else:
            produced = [(name, shard_tensor(name, tensor, rank, world, num_kv_heads))]
        for key, value in produced:
            value = _cast(key, value, dtype)
            info = _merge_info(key)
            if info is None:
                yield from out(key, value)
                continue
            merged_key, slot, slots = info
            group = merge_buf.setdefault(merged_key, {})
            group[slot] = value
            if all(s in group for s in slots):
                del merge_buf[merged_key]
                yield from out(merged_key, torch.cat([group[s] for s in slots], dim=0))
    if merge_buf:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"incomplete merge groups in checkpoint: {sorted(merge_buf)}")
    if expert_buf:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"incomplete expert tensors in checkpoint: {sorted(expert_buf)}")


def load_w8a8_state_dict(items: Iterable[Tuple[str, torch.Tensor]], rank: int, world: int,
                         num_kv_heads: Optional[int], quantise: Optional[Quantiser] = None,
                         device: Optional[torch.device] = None,
                         dtype: torch.dtype = torch.bfloat16,
                         num_experts: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """``dict(w8a8_weight_stream(...))`` -- the state dict to hand to the
    model's ``load_state_dict`` in place of the engine's
    ``{k: v.to(dtype) for k, v in load_weight(...)}`` (M/engine/engine.py:139-146)."""
    return dict(w8a8_weight_stream(items, rank, world, num_kv_heads, quantise, device, dtype, num_experts))
