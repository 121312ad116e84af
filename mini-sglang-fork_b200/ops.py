"""Torch-facing wrappers of the C ABI (``include/w8a8_tp.h``).

Every op launches hand-written sm_100a CUDA through ``_w8a8_tp.so`` on the
caller's current CUDA stream.  There is no CPU or library fallback: a
non-CUDA tensor, a missing library or a non-B200 device raises.
"""
from __future__ import annotations

import ctypes
from typing import Dict, NamedTuple, Optional, Tuple

import torch

from . import _lib

__all__ = [
    "quant_per_token",
    "silu_and_mul_quant",
    "silu_and_mul",
    "w8a8_gemm",
    "gate_up_silu_quant",
    "gemm_silu",
    "quant_rows_amax",
    "gemm_plan",
    "gemm_workspace",
    "device_error",
    "reset_gemm_workspace",
    "check_gemm_operands",
    "QuantizedActivation",
    "WORKSPACE_BYTES",
    "MoeRouting",
    "moe_align",
    "moe_quant_scatter",
    "moe_gemm",
    "moe_quant_rows",
    "moe_sum",
    "fused_experts_w8a8",
]

# Split-K workspace kept per device (zeroed once, left zeroed by every call).
WORKSPACE_BYTES = 64 << 20
_workspaces: Dict[int, torch.Tensor] = {}


class QuantizedActivation:
    """An int8 activation with its per-token fp32 scales (``q [M, K]``, ``s [M]``).

    Produced by :func:`silu_and_mul_quant` and accepted by every W8A8 linear's
    ``forward`` in place of a bf16 tensor, so ``GatedMLP`` can hand the fused
    SiLU*mul+quant output straight to ``down_proj``.
    """

    __slots__ = ("q", "s")

    def __init__(self, q: torch.Tensor, s: torch.Tensor):
        self.q = q
        self.s = s

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(name: str, *ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise _lib.W8A8Error(_lib.ERR_UNSUPPORTED,
                                 f"{name}: CUDA tensors required (got {t.device}); there is no CPU path")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def gemm_workspace(device: torch.device) -> torch.Tensor:
    """The zero-initialised split-K workspace of ``device`` (allocated once)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None:
        ws = torch.zeros(WORKSPACE_BYTES, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws


def quant_per_token(x: torch.Tensor, out_q: Optional[torch.Tensor] = None,
                    out_s: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-token symmetric absmax int8 quantisation of ``x [M, K]`` bf16."""
    _require_cuda("quant_per_token", x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "quant_per_token: x must be a 2-D bf16 tensor with unit column stride")
    m, k = x.shape
    q = out_q if out_q is not None else torch.empty(m, k, dtype=torch.int8, device=x.device)
    s = out_s if out_s is not None else torch.empty(m, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    _lib.check(lib.w8a8_quant_per_token(_ptr(x), x.stride(0), _ptr(q), _ptr(s), m, k, _stream(x)),
               "quant_per_token")
    return q, s


def silu_and_mul_quant(gate_up: torch.Tensor, with_bf16: bool = False):
    """Fused ``silu(g) * u`` (rounded to bf16) + per-token int8 quantisation.

    ``gate_up [M, 2I]`` bf16 -> :class:`QuantizedActivation` (``q [M, I]``,
    ``s [M]``); with ``with_bf16`` also returns the bf16 ``[M, I]`` product.
    """
    _require_cuda("silu_and_mul_quant", gate_up)
    if gate_up.dtype != torch.bfloat16 or gate_up.dim() != 2 or gate_up.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "silu_and_mul_quant: gate_up must be 2-D bf16 with unit column stride")
    m, two_i = gate_up.shape
    if two_i % 2:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "silu_and_mul_quant: last dim must be even")
    i = two_i // 2
    q = torch.empty(m, i, dtype=torch.int8, device=gate_up.device)
    s = torch.empty(m, dtype=torch.float32, device=gate_up.device)
    y = torch.empty(m, i, dtype=torch.bfloat16, device=gate_up.device) if with_bf16 else None
    lib = _lib.load()
    _lib.check(lib.w8a8_silu_mul_quant(_ptr(gate_up), gate_up.stride(0), _ptr(q), _ptr(s), _ptr(y), m, i,
                                       _stream(gate_up)), "silu_and_mul_quant")
    qa = QuantizedActivation(q, s)
    return (qa, y) if with_bf16 else qa


def rmsnorm_quant(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
                  with_bf16: bool = False):
    """RMSNorm (after ``x + residual`` when a residual is given, updating the
    residual in place, as ``fused_add_rmsnorm`` does) fused with the per-token
    quantiser.  Returns ``(QuantizedActivation, residual)`` -- the residual is
    ``x`` itself without one (M/layers/norm.py:31-38) -- plus the bf16
    normalised rows with ``with_bf16``."""
    _require_cuda("rmsnorm_quant", x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "rmsnorm_quant: x must be 2-D bf16 with unit column stride")
    m, k = x.shape
    if weight.dtype != torch.bfloat16 or weight.shape != (k,) or not weight.is_contiguous():
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "rmsnorm_quant: weight must be a contiguous bf16 [K] vector")
    if residual is not None and (residual.dtype != torch.bfloat16 or residual.shape != x.shape
                                 or residual.stride(1) != 1):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "rmsnorm_quant: residual must match x (bf16, unit column stride)")
    q = torch.empty(m, k, dtype=torch.int8, device=x.device)
    s = torch.empty(m, dtype=torch.float32, device=x.device)
    y = torch.empty(m, k, dtype=torch.bfloat16, device=x.device) if with_bf16 else None
    lib = _lib.load()
    _lib.check(lib.w8a8_rmsnorm_quant(_ptr(x), x.stride(0), _ptr(residual),
                                      residual.stride(0) if residual is not None else k, _ptr(weight), float(eps),
                                      _ptr(q), _ptr(s), _ptr(residual), _ptr(y), m, k, _stream(x)),
               "rmsnorm_quant")
    qa = QuantizedActivation(q, s)
    res = residual if residual is not None else x
    return (qa, res, y) if with_bf16 else (qa, res)


def silu_and_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 ``silu(x[:, :I]) * x[:, I:]`` — the signature of ``silu_and_mul``
    (M/layers/activation.py:9-12).  The bf16-only form of the SiLU*mul kernel:
    no quantisation, the product written straight into ``out`` (allocated
    when None)."""
    _require_cuda("silu_and_mul", x, out)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1 or x.shape[1] % 2:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "silu_and_mul: x must be 2-D bf16 [M, 2I], unit column stride")
    m, i = x.shape[0], x.shape[1] // 2
    if out is None:
        out = torch.empty(m, i, dtype=torch.bfloat16, device=x.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (m, i) or not out.is_contiguous():
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "silu_and_mul: out must be contiguous bf16 [M, I]")
    _lib.check(_lib.load().w8a8_silu_mul_quant(_ptr(x), x.stride(0), None, None, _ptr(out), m, i, _stream(x)),
               "silu_and_mul")
    return out


def gemm_plan(m: int, n: int, k: int, variant: int = 0, ctas: int = 0,
              workspace_bytes: int = WORKSPACE_BYTES, num_sms: int = 148) -> Dict[str, int]:
    """Host-only query of the tile configuration the GEMM would use."""
    out = (ctypes.c_int64 * 8)()
    _lib.check(_lib.load().w8a8_gemm_plan(m, n, k, variant, ctas, workspace_bytes, num_sms, out),
               "gemm_plan")
    keys = ("variant", "bn", "swap", "tiles", "grid", "kblocks", "gran", "workspace_bytes")
    return dict(zip(keys, (int(v) for v in out)))


def check_gemm_operands(name: str, aq: torch.Tensor, wq: torch.Tensor, sa: torch.Tensor, sw: torch.Tensor,
                        bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                        out_i32: Optional[torch.Tensor] = None,
                        alloc_out: bool = True) -> Tuple[int, int, int, Optional[torch.Tensor]]:
    """Host-side validation shared by every GEMM entry (plain and fused): all
    tensors on one CUDA device, int8 2-D operands with matching K, fp32 scale
    vectors of exactly M and N elements, bf16 bias [N], bf16 out [M, N]
    (allocated when None), int32 out_i32 [M, N].  A bad operand raises here,
    before any pointer reaches a kernel (a host pointer or a short scale
    vector would otherwise be read by the GPU).  Returns (M, N, K, out); out
    stays None with ``alloc_out=False``."""
    if aq.dtype != torch.int8 or wq.dtype != torch.int8 or aq.dim() != 2 or wq.dim() != 2:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: 2-D int8 operands required")
    if not (aq.is_contiguous() and wq.is_contiguous() and sa.is_contiguous() and sw.is_contiguous()):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: contiguous operands required")
    if sa.dtype != torch.float32 or sw.dtype != torch.float32:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: fp32 scales required")
    m, k = aq.shape
    n, k2 = wq.shape
    if k2 != k or sa.numel() != m or sw.numel() != n:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG,
                             f"{name}: shape mismatch A{tuple(aq.shape)} B{tuple(wq.shape)} "
                             f"sa[{sa.numel()}] sw[{sw.numel()}]")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: bias must be contiguous bf16 [N]")
    if out is not None and (out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or not out.is_contiguous()):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: out must be contiguous bf16 [M, N]")
    if out_i32 is not None and (out_i32.dtype != torch.int32 or tuple(out_i32.shape) != (m, n)
                                or not out_i32.is_contiguous()):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: out_i32 must be contiguous int32 [M, N]")
    _require_cuda(name, aq, wq, sa, sw, bias, out, out_i32)
    devs = {t.device for t in (aq, wq, sa, sw, bias, out, out_i32) if t is not None}
    if len(devs) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: operands on several devices {sorted(map(str, devs))}")
    if out is None and alloc_out:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=aq.device)
    return m, n, k, out


def w8a8_gemm(aq: torch.Tensor, wq: torch.Tensor, sa: torch.Tensor, sw: torch.Tensor,
              bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              out_i32: Optional[torch.Tensor] = None, variant: int = 0, ctas: int = 0) -> torch.Tensor:
    """``bf16((f32(aq @ wq.T) * sa[:, None]) * sw[None, :] + bias)`` on tcgen05.

    ``aq [M, K]`` int8, ``wq [N, K]`` int8, ``sa [M]`` / ``sw [N]`` fp32,
    ``bias [N]`` bf16 or None.  ``out_i32`` (optional ``[M, N]`` int32)
    receives the exact accumulator.  ``variant`` / ``ctas`` override the
    planner (0 = automatic).
    """
    m, n, k, out = check_gemm_operands("w8a8_gemm", aq, wq, sa, sw, bias, out, out_i32)
    ws = gemm_workspace(aq.device)
    lib = _lib.load()
    st = lib.w8a8_gemm_config(_ptr(aq), _ptr(wq), _ptr(sa), _ptr(sw), _ptr(bias), _ptr(out), _ptr(out_i32),
                              m, n, k, variant, ctas, _ptr(ws), ws.numel(), _stream(aq))
    _lib.check(st, "w8a8_gemm")
    return out


def gemm_silu(aq: torch.Tensor, wq: torch.Tensor, sa: torch.Tensor, sw: torch.Tensor,
              bias: Optional[torch.Tensor] = None) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """The gate_up GEMM with SiLU*mul in its epilogue: ``wq [2I, K]`` is the
    merged [gate; up] weight; returns ``(y, amax)`` with ``y = bf16(silu(g) *
    u)`` ``[M, I]`` (g, u the bf16 values :func:`w8a8_gemm` would write) and
    ``amax [M]`` int32 holding the float bits of every row's max |y|.  None
    where the fusion does not apply (M <= 128 or 2I % 256 != 0: the 2-SM pair
    kernel carries the SiLU epilogue)."""
    m, n2, k, _ = check_gemm_operands("gemm_silu", aq, wq, sa, sw, bias, alloc_out=False)
    if m <= 128 or n2 % 256:
        return None
    dev = aq.device
    y = torch.empty(m, n2 // 2, dtype=torch.bfloat16, device=dev)
    amax = torch.zeros(m, dtype=torch.int32, device=dev)  # raised atomically by the epilogue
    ws = gemm_workspace(dev)
    lib = _lib.load()
    st = lib.w8a8_gemm_silu(_ptr(aq), _ptr(wq), _ptr(sa), _ptr(sw), _ptr(bias), _ptr(y), _ptr(amax),
                            m, n2, k, _ptr(ws), ws.numel(), _stream(aq))
    if st == _lib.ERR_UNSUPPORTED:
        return None
    _lib.check(st, "gemm_silu")
    return y, amax


def quant_rows_amax(y: torch.Tensor, amax: torch.Tensor) -> QuantizedActivation:
    """Per-token quantisation of ``y [M, K]`` bf16 whose row absmax is already
    known (``amax [M]``, float bits as :func:`gemm_silu` leaves them); the same
    rule as :func:`quant_per_token`."""
    _require_cuda("quant_rows_amax", y, amax)
    if y.dtype != torch.bfloat16 or y.dim() != 2 or y.stride(1) != 1 or amax.numel() != y.shape[0]:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "quant_rows_amax: y must be 2-D bf16, amax [M]")
    m, k = y.shape
    q = torch.empty(m, k, dtype=torch.int8, device=y.device)
    s = torch.empty(m, dtype=torch.float32, device=y.device)
    lib = _lib.load()
    _lib.check(lib.w8a8_quant_rows_amax(_ptr(y), y.stride(0), _ptr(amax), _ptr(q), _ptr(s), m, k, _stream(y)),
               "quant_rows_amax")
    return QuantizedActivation(q, s)


def gate_up_silu_quant(aq: torch.Tensor, wq: torch.Tensor, sa: torch.Tensor, sw: torch.Tensor,
                       bias: Optional[torch.Tensor] = None, with_bf16: bool = False):
    """gate_up GEMM, SiLU*mul and per-token quantisation with the [M, 2I]
    gate_up tensor never in HBM (:func:`gemm_silu`, then
    :func:`quant_rows_amax`).  Bit-identical to
    ``silu_and_mul_quant(w8a8_gemm(...))``.  Returns None where the fusion
    does not apply; with ``with_bf16`` returns ``(QuantizedActivation, y)``."""
    r = gemm_silu(aq, wq, sa, sw, bias)
    if r is None:
        return None
    y, amax = r
    qa = quant_rows_amax(y, amax)
    return (qa, y) if with_bf16 else qa


# ---------------------------------------------------------------------------
# mixture of experts (fused_experts_impl, M/moe/fused.py:135-215)
# ---------------------------------------------------------------------------
class MoeRouting(NamedTuple):
    """The expert-sorted layout of one batch's routed slots (``w8a8_moe_align``).

    Slot ``s = t * topk + j`` is token t's j-th choice.  Rows ``[0, 128 *
    num_blocks)`` of every sorted buffer are in use (``num_blocks`` lives on
    the device); ``P = 128 * max_blocks`` rows are allocated."""
    sorted_ids: torch.Tensor    # [P] int32: slot of each row (num_slots on padding)
    block_expert: torch.Tensor  # [max_blocks] int32: expert of each 128-row block
    num_blocks: torch.Tensor    # [1] int32, device
    inv_pos: torch.Tensor       # [num_slots] int32: row of each slot (-1: dropped)
    sa_sorted: torch.Tensor     # [P] fp32: activation scale of each row (0 on padding)
    max_blocks: int
    num_experts: int
    topk: int


def _one_device(name: str, *ts: Optional[torch.Tensor]) -> None:
    devs = {t.device for t in ts if t is not None}
    if len(devs) > 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"{name}: operands on several devices {sorted(map(str, devs))}")


def _check_2d(name: str, t: torch.Tensor, dtype: torch.dtype, shape: Tuple[int, ...]) -> None:
    if t.dtype != dtype or tuple(t.shape) != tuple(shape) or not t.is_contiguous():
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG,
                             f"{name}: expected a contiguous {dtype} tensor of shape {tuple(shape)}, got "
                             f"{t.dtype} {tuple(t.shape)}{'' if t.is_contiguous() else ' (non-contiguous)'}")


def moe_align(topk_ids: torch.Tensor, num_experts: int) -> MoeRouting:
    """``moe_align_block_size`` (M/moe/fused.py:32-83) with 128-row blocks."""
    _require_cuda("moe_align", topk_ids)
    if topk_ids.dim() != 2 or topk_ids.dtype != torch.int32 or not topk_ids.is_contiguous():
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "moe_align: topk_ids must be a contiguous int32 [T, topk]")
    t, k = topk_ids.shape
    n = t * k
    lib = _lib.load()
    mb = int(lib.w8a8_moe_max_blocks(n, num_experts)) if n > 0 else 0
    dev = topk_ids.device
    p = 128 * mb
    r = MoeRouting(torch.empty(p, dtype=torch.int32, device=dev), torch.empty(max(mb, 1), dtype=torch.int32, device=dev),
                   torch.empty(1, dtype=torch.int32, device=dev), torch.empty(n, dtype=torch.int32, device=dev),
                   torch.empty(p, dtype=torch.float32, device=dev), mb, num_experts, k)
    _lib.check(lib.w8a8_moe_align(_ptr(topk_ids), n, num_experts, _ptr(r.sorted_ids), _ptr(r.block_expert),
                                  _ptr(r.num_blocks), _ptr(r.inv_pos), _ptr(r.sa_sorted), _stream(topk_ids)),
               "moe_align")
    return r


def moe_quant_scatter(x: torch.Tensor, routing: MoeRouting) -> torch.Tensor:
    """Per-token quantisation of ``x [T, H]`` into the expert-sorted rows:
    returns ``q_sorted [P, H]`` int8 and fills ``routing.sa_sorted``."""
    _require_cuda("moe_quant_scatter", x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "moe_quant_scatter: x must be a 2-D bf16 tensor with unit column stride")
    t, h = x.shape
    _one_device("moe_quant_scatter", x, routing.inv_pos, routing.sa_sorted)
    if routing.inv_pos.numel() != t * routing.topk:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "moe_quant_scatter: routing was built for another token count")
    q = torch.empty(128 * routing.max_blocks, h, dtype=torch.int8, device=x.device)
    if t > 0:
        _lib.check(_lib.load().w8a8_moe_quant_scatter(_ptr(x), x.stride(0), t, h, _ptr(routing.inv_pos), routing.topk,
                                                      _ptr(q), _ptr(routing.sa_sorted), _stream(x)),
                   "moe_quant_scatter")
    return q


def moe_gemm(a_sorted: torch.Tensor, sa_sorted: torch.Tensor, w: torch.Tensor, sw: torch.Tensor,
             routing: MoeRouting, route_w: Optional[torch.Tensor] = None, silu: bool = False):
    """Grouped W8A8 GEMM over the expert-sorted rows (``w8a8_moe_gemm``):
    ``w [E, N, K]`` int8, ``sw [E, N]`` fp32.  ``silu``: ``w`` is [gate; up]
    per expert and the result is ``(y [P, N/2] bf16, amax [P] int32)``;
    otherwise ``c [P, N]`` bf16 with the routing weight (``route_w [T, topk]``
    fp32, nullable) applied."""
    _require_cuda("moe_gemm", a_sorted, sa_sorted, w, sw, route_w)
    e, n, k = w.shape if w.dim() == 3 else (0, 0, 0)
    p = 128 * routing.max_blocks
    if w.dim() != 3 or e != routing.num_experts:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"moe_gemm: w must be [E={routing.num_experts}, N, K]")
    _one_device("moe_gemm", a_sorted, sa_sorted, w, sw, route_w, routing.sorted_ids, routing.block_expert)
    _check_2d("moe_gemm w", w, torch.int8, (e, n, k))
    _check_2d("moe_gemm sw", sw, torch.float32, (e, n))
    _check_2d("moe_gemm a_sorted", a_sorted, torch.int8, (p, k))
    _check_2d("moe_gemm sa_sorted", sa_sorted, torch.float32, (p,))
    if route_w is not None:
        _check_2d("moe_gemm route_w", route_w, torch.float32, (routing.inv_pos.numel() // routing.topk, routing.topk))
        if silu:
            raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "moe_gemm: no routing weight with the SiLU epilogue")
    dev = a_sorted.device
    out = torch.empty(p, n // 2 if silu else n, dtype=torch.bfloat16, device=dev)
    amax = torch.zeros(p, dtype=torch.int32, device=dev) if silu else None
    if p > 0:
        _lib.check(_lib.load().w8a8_moe_gemm(
            _ptr(a_sorted), _ptr(w), _ptr(sa_sorted), _ptr(sw), _ptr(routing.block_expert), _ptr(routing.num_blocks),
            routing.max_blocks, _ptr(routing.sorted_ids), _ptr(route_w), routing.inv_pos.numel(), _ptr(out),
            _ptr(amax), e, n, k, _stream(a_sorted)), "moe_gemm")
    return (out, amax) if silu else out


def moe_quant_rows(y: torch.Tensor, amax: torch.Tensor, routing: MoeRouting) -> QuantizedActivation:
    """Row quantisation of the sorted ``y [P, I]`` with its known absmax, over
    the rows in use only."""
    _require_cuda("moe_quant_rows", y, amax)
    p = 128 * routing.max_blocks
    if y.dtype != torch.bfloat16 or y.dim() != 2 or y.shape[0] != p or y.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "moe_quant_rows: y must be a bf16 [P, I] tensor")
    _check_2d("moe_quant_rows amax", amax, torch.int32, (p,))
    _one_device("moe_quant_rows", y, amax, routing.num_blocks)
    i = y.shape[1]
    q = torch.empty(p, i, dtype=torch.int8, device=y.device)
    s = torch.empty(p, dtype=torch.float32, device=y.device)
    if p > 0:
        _lib.check(_lib.load().w8a8_moe_quant_rows(_ptr(y), y.stride(0), _ptr(amax), _ptr(q), _ptr(s),
                                                   _ptr(routing.num_blocks), routing.max_blocks, i, _stream(y)),
                   "moe_quant_rows")
    return QuantizedActivation(q, s)


def moe_sum(c_sorted: torch.Tensor, routing: MoeRouting, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``moe_sum_reduce`` (M/kernel/triton/fused_moe.py:5-48): ``out[t] =
    bf16(sum_j f32(c[row(t, j)]))`` in choice order."""
    _require_cuda("moe_sum", c_sorted, out)
    t = routing.inv_pos.numel() // max(routing.topk, 1)
    _one_device("moe_sum", c_sorted, out, routing.inv_pos)
    if c_sorted.dtype != torch.bfloat16 or c_sorted.dim() != 2 or c_sorted.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "moe_sum: c_sorted must be a bf16 [P, H] tensor")
    h = c_sorted.shape[1]
    if out is None:
        out = torch.empty(t, h, dtype=torch.bfloat16, device=c_sorted.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (t, h) or out.stride(1) != 1:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, f"moe_sum: out must be bf16 [{t}, {h}] with unit column stride")
    if t > 0:
        _lib.check(_lib.load().w8a8_moe_sum(_ptr(c_sorted), c_sorted.stride(0), _ptr(routing.inv_pos), t,
                                            routing.topk, h, _ptr(out), out.stride(0), _stream(c_sorted)), "moe_sum")
    return out


def fused_experts_w8a8(x: torch.Tensor, w1q: torch.Tensor, sw1: torch.Tensor, w2q: torch.Tensor,
                       sw2: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The W8A8 counterpart of ``fused_experts_impl`` (M/moe/fused.py:135-215)
    with ``activation="silu"`` and the routing weight applied to the down
    GEMM: ``x [T, H]`` bf16, ``w1q [E, 2I, H]`` / ``sw1 [E, 2I]``, ``w2q [E,
    H, I]`` / ``sw2 [E, H]``, ``topk_weights [T, k]`` fp32, ``topk_ids [T, k]``
    int32 -> ``[T, H]`` bf16.  Six launches, no host sync: align, quantise
    into the sorted rows, gate_up grouped GEMM with SiLU*mul, quantise y,
    down grouped GEMM with the routing weight, top-k sum."""
    _require_cuda("fused_experts_w8a8", x, w1q, sw1, w2q, sw2, topk_weights, topk_ids)
    if x.dim() != 2 or w1q.dim() != 3 or w2q.dim() != 3:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "fused_experts_w8a8: x [T, H], w1q [E, 2I, H], w2q [E, H, I]")
    t, h = x.shape
    e, n2, _ = w1q.shape
    if tuple(w1q.shape) != (e, n2, h) or tuple(w2q.shape) != (e, h, n2 // 2) or n2 % 2:
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG,
                             f"fused_experts_w8a8: w1q {tuple(w1q.shape)} / w2q {tuple(w2q.shape)} do not match "
                             f"H={h}")
    if topk_ids.dim() != 2 or topk_ids.shape[0] != t or tuple(topk_weights.shape) != tuple(topk_ids.shape):
        raise _lib.W8A8Error(_lib.ERR_INVALID_ARG, "fused_experts_w8a8: topk_ids / topk_weights must be [T, topk]")
    _check_2d("fused_experts_w8a8 topk_weights", topk_weights, torch.float32, tuple(topk_ids.shape))
    _one_device("fused_experts_w8a8", x, w1q, sw1, w2q, sw2, topk_weights, topk_ids, out)
    routing = moe_align(topk_ids, e)
    if out is None:
        out = torch.empty(t, h, dtype=torch.bfloat16, device=x.device)
    if routing.max_blocks == 0:
        return out.zero_()
    qx = moe_quant_scatter(x, routing)
    y, amax = moe_gemm(qx, routing.sa_sorted, w1q, sw1, routing, silu=True)
    qy = moe_quant_rows(y, amax, routing)
    c3 = moe_gemm(qy.q, qy.s, w2q, sw2, routing, route_w=topk_weights)
    return moe_sum(c3, routing, out)


# The stream-K counter region at the head of a GEMM workspace (65536 tile
# counters, csrc/gemm_plan.h kCounterBytes).
_COUNTER_BYTES = 65536 * 4


def reset_gemm_workspace(device: Optional[torch.device] = None) -> None:
    """Zero the stream-K tile counters of the workspace(s) on the caller's
    stream.  A successful GEMM leaves its counters at zero, but a call whose
    bounded wait gave up can stop before resetting the counters of its cut
    tiles; :func:`device_error` calls this whenever it clears a non-zero error
    word, so the next call starts from zero counters."""
    for idx, ws in _workspaces.items():
        if device is None or device.index in (None, idx):
            ws[:_COUNTER_BYTES].zero_()


def device_error(clear: bool = True) -> int:
    """Device-side error bits (bounded waits that gave up); synchronises.
    Clearing a non-zero word also resets the GEMM workspaces' counters."""
    code = ctypes.c_int(0)
    _lib.check(_lib.load().w8a8_device_error(ctypes.byref(code), 1 if clear else 0), "device_error")
    if clear and code.value != 0:
        reset_gemm_workspace()
        torch.cuda.synchronize()
    return code.value
