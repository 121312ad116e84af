"""Benchmark of the W8A8 tensor-parallel linear path on B200.

Workload: the four quantised linears of one Qwen3-32B
decoder layer at TP = N -- qkv (column-parallel) -> o_proj (row-parallel +
all-reduce) -> gate_up (column-parallel) -> fused SiLU*mul + per-token quant
-> down (row-parallel + all-reduce).  Attention is not part of the path: the
q slice of the qkv output stands in for the attention output that feeds
o_proj.  hidden 5120, 64 q / 8 kv heads x 128, intermediate 25600.  A step is
one pass of that stack over M tokens (headline M = 4096, the prefill chunk;
the decode sizes M = 1, 32, 128, 256 are reported in ``sweep``).

Synthetic seeded data: activations ~N(0, 1) bf16; a synthetic bf16
checkpoint (~N(0, 0.02) per projection, q/k/v/o/gate/up/down, the same on
every rank) goes through the package's own loader, which quantises each
UNSHARDED weight per output channel and shards and merges it exactly as the
reference's loader shards bf16 weights -- so the benchmarked layers are the
ones a real load builds.

After timing, the same layers' outputs on a fixed sample of rows are checked
against the CPU oracle at every N (``parity``), a per-op breakdown is timed
(``breakdown_us``), and at N > 1 the row-parallel reduce is also run through
the reference's own NCCL path -- ``ncclMemAlloc`` + symmetric window +
``ncclAllReduce`` with the copies in and out (``nccl_baseline``).

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 launch one rank per GPU with torchrun (RANK / WORLD_SIZE from env).
Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import copy
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# BASELINE configs 2-4; cfg3 (the headline the driver runs) is the default.
WORKLOADS = {
    "cfg3": {"hidden": 5120, "head_dim": 128, "nq": 64, "nkv": 8, "inter": 25600, "layers": 1, "mlp_only": False,
             "m": 4096, "sweep": [1, 32, 128, 256],
             "metric": "W8A8 TP-layer tokens/s (Qwen3-32B decoder-layer linears: qkv, o_proj+AR, gate_up, "
                       "silu*mul+quant, down+AR)",
             "desc": "cfg3 Qwen3-32B decoder-layer W8A8 linears, TP=N, headline M = prefill chunk"},
    "cfg2": {"hidden": 4096, "head_dim": 128, "nq": 32, "nkv": 8, "inter": 12288, "layers": 1, "mlp_only": True,
             "m": 8192, "sweep": [1, 16, 64, 256, 2048],
             "metric": "W8A8 MLP tokens/s (Qwen3-8B GatedMLP: gate_up, silu*mul+quant, down)",
             "desc": "cfg2 Qwen3-8B W8A8 MLP block (gate_up 4096->24576, silu*mul+quant, down 12288->4096)"},
    "cfg4": {"hidden": 8192, "head_dim": 128, "nq": 64, "nkv": 8, "inter": 28672, "layers": 4, "mlp_only": False,
             "m": 8192, "sweep": [256],
             "metric": "W8A8 TP-layer tokens/s (Llama-3.1-70B, 4 consecutive decoder layers' linears with fused "
                       "row-parallel all-reduce)",
             "desc": "cfg4 Llama-3.1-70B 4-layer W8A8 linear stack, TP=N"},
}
WORKLOAD = "cfg3"
HIDDEN, HEAD_DIM, NQ, NKV, INTER, LAYERS, MLP_ONLY = 5120, 128, 64, 8, 25600, 1, False
METRIC = WORKLOADS["cfg3"]["metric"]
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20
INT8_NOMINAL_TOPS = 4500.0
L2_NOTE = ("flushed before every timed step (256 MB written, then read back so no dirty line is left); "
           "per-step CUDA-event timing of a CUDA-graph replay")

# The synthetic checkpoint of one decoder layer: projection -> (module, N, K).
PROJ = {
    "q_proj": ("self_attn", NQ * HEAD_DIM, HIDDEN),
    "k_proj": ("self_attn", NKV * HEAD_DIM, HIDDEN),
    "v_proj": ("self_attn", NKV * HEAD_DIM, HIDDEN),
    "o_proj": ("self_attn", HIDDEN, NQ * HEAD_DIM),
    "gate_proj": ("mlp", INTER, HIDDEN),
    "up_proj": ("mlp", INTER, HIDDEN),
    "down_proj": ("mlp", HIDDEN, INTER),
}
PREFIX = "model.layers.0."


def _proj_table():
    return {
        "q_proj": ("self_attn", NQ * HEAD_DIM, HIDDEN),
        "k_proj": ("self_attn", NKV * HEAD_DIM, HIDDEN),
        "v_proj": ("self_attn", NKV * HEAD_DIM, HIDDEN),
        "o_proj": ("self_attn", HIDDEN, NQ * HEAD_DIM),
        "gate_proj": ("mlp", INTER, HIDDEN),
        "up_proj": ("mlp", INTER, HIDDEN),
        "down_proj": ("mlp", HIDDEN, INTER),
    }


def select_workload(name: str) -> None:
    """Rebind the module's workload shape (3 or 4)."""
    global WORKLOAD, HIDDEN, HEAD_DIM, NQ, NKV, INTER, LAYERS, MLP_ONLY, METRIC, PROJ
    w = WORKLOADS[name]
    WORKLOAD = name
    HIDDEN, HEAD_DIM, NQ, NKV, INTER = w["hidden"], w["head_dim"], w["nq"], w["nkv"], w["inter"]
    LAYERS, MLP_ONLY, METRIC = w["layers"], w["mlp_only"], w["metric"]
    PROJ = _proj_table()


def _pkg():
    return importlib.import_module("mini-sglang-fork_b200")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def local_shapes(tp: int):
    """Per-rank (N, K) of qkv, o_proj, gate_up, down (M/layers/linear.py:56-127);
    gate_up and down only for an MLP-only workload."""
    lq = NQ // tp
    lkv = max(1, NKV // tp)
    sh = {
        "qkv": ((lq + 2 * lkv) * HEAD_DIM, HIDDEN),
        "o_proj": (HIDDEN, NQ * HEAD_DIM // tp),
        "gate_up": (2 * INTER // tp, HIDDEN),
        "down": (HIDDEN, INTER // tp),
    }
    if MLP_ONLY:
        del sh["qkv"], sh["o_proj"]
    return sh


def layer_ops(tp: int):
    """Integer ops (2*M*N*K summed) and weight bytes of all the step's linears per token."""
    sh = local_shapes(tp)
    ops_per_token = LAYERS * sum(2 * n * k for n, k in sh.values())
    wbytes = LAYERS * sum(n * k + 4 * n for n, k in sh.values())
    return ops_per_token, wbytes


def workload_config(world: int, m: int):
    """The workload keys both arms (GPU and the CPU reference) report."""
    return {"workload": WORKLOADS[WORKLOAD]["desc"], "M": m, "hidden": HIDDEN, "heads": [NQ, NKV],
            "head_dim": HEAD_DIM, "intermediate": INTER, "layers": LAYERS, "parallelism": f"tp{world}"}


def full_weight(name: str, dev: torch.device, layer: int = 0) -> torch.Tensor:
    """The synthetic bf16 checkpoint tensor of one projection of one layer
    (identical on every rank)."""
    _, n, k = PROJ[name]
    g = torch.Generator(device=dev).manual_seed(1000 + 16 * layer + list(PROJ).index(name))
    return (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()


def checkpoint_items(dev: torch.device):
    """(name, tensor) pairs as safetensors yields them, one projection at a time."""
    for layer in range(LAYERS):
        for name, (module, _, _) in PROJ.items():
            if MLP_ONLY and module != "mlp":
                continue
            yield f"model.layers.{layer}.{module}.{name}.weight", full_weight(name, dev, layer)


DECODE_CHAIN = 8  # decode steps per graph replay in the sweep


def clone_layers(layers):
    """Copies of a stack's layers with their own weight storage (same values)."""
    out = []
    for lay in layers:
        new = {}
        for name, layer in lay.items():
            c = copy.copy(layer)
            c.weight = layer.weight.clone()
            c.weight_scale = layer.weight_scale.clone()
            new[name] = c
        out.append(new)
    return out


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, out_dir: str):
        self.proc = None
        self.path = os.path.join(out_dir, f"clocks_rank{device_index}.csv")
        target = str(device_index)
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            target = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            pass
        self.target = target

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.target, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
                except ValueError:
                    continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        load = [r for r in rows if r[2] > 250.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in load:
            for nm, flag in zip(names, r[3][1:]):
                if flag.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(load),
                "power_w_max": max(r[2] for r in rows)}


# --------------------------------------------------------------------------- the layer stack
class Stack:
    """The workload's W8A8 linears on this rank (LAYERS decoder layers of
    qkv, o_proj, gate_up, down -- or gate_up, down only), built through the
    package's public layer classes and loaded from the synthetic checkpoint
    with the package's loader (quantise unsharded, then shard)."""

    def __init__(self, pkg, tp: int, rank: int, dev: torch.device):
        L = pkg.layers
        self.pkg = pkg
        self.layers = []
        for _ in range(LAYERS):
            lay = {}
            if not MLP_ONLY:
                lay["qkv"] = L.LinearQKVMerged(HIDDEN, HEAD_DIM, NQ, NKV, has_bias=False)
                lay["o_proj"] = L.LinearOProj(NQ * HEAD_DIM, HIDDEN, has_bias=False)
            lay["gate_up"] = L.LinearColParallelMerged(HIDDEN, [INTER, INTER], has_bias=False)
            lay["down"] = L.LinearRowParallel(INTER, HIDDEN, has_bias=False)
            self.layers.append(lay)
        self.q_cols = (NQ // tp) * HEAD_DIM
        state = pkg.load_w8a8_state_dict(checkpoint_items(dev), rank, tp, NKV, device=dev)
        keys = {"qkv": "self_attn.qkv_proj", "o_proj": "self_attn.o_proj", "gate_up": "mlp.gate_up_proj",
                "down": "mlp.down_proj"}
        for i, lay in enumerate(self.layers):
            for name, layer in lay.items():
                key = f"model.layers.{i}.{keys[name]}"
                layer.load_state_dict({"weight": state.pop(f"{key}.weight"),
                                       "weight_scale": state.pop(f"{key}.weight_scale")})
        assert not state, sorted(state)
        first = self.layers[0]
        self.qkv, self.o_proj = first.get("qkv"), first.get("o_proj")
        self.gate_up, self.down = first["gate_up"], first["down"]
        torch.cuda.synchronize()

    def _layer(self, lay, x: torch.Tensor) -> torch.Tensor:
        if not MLP_ONLY:
            qkv = lay["qkv"].forward(x)
            x = lay["o_proj"].forward(qkv[:, : self.q_cols])
        return lay["down"].forward(lay["gate_up"].forward_silu_quant(x))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.forward_layers(self.layers, x)

    def forward_layers(self, layers, x: torch.Tensor) -> torch.Tensor:
        for lay in layers:
            x = self._layer(lay, x)
        return x

    def forward_traced(self, x: torch.Tensor):
        """The first layer's forward, keeping every linear's input and output
        (parity check; decoder layers only)."""
        t = {"x": x}
        t["qkv"] = self.qkv.forward(x)
        t["attn"] = t["qkv"][:, : self.q_cols]
        t["h"] = self.o_proj.forward(t["attn"])
        t["gu"] = self.gate_up.forward(t["h"])  # the gate_up GEMM alone, checked on its own
        qa = self.gate_up.forward_silu_quant(t["h"])  # the timed path (SiLU in the GEMM's epilogue)
        t["q"], t["s"] = qa.q, qa.s
        t["out"] = self.down.forward(qa)
        return t

    def forward_nccl(self, x: torch.Tensor, nccl) -> torch.Tensor:
        """The same stack with the row-parallel reduce through ``nccl`` (the
        reference's path: GEMM, then an all-reduce call) instead of fused."""
        ops = self.pkg.ops
        for lay in self.layers:
            if not MLP_ONLY:
                qkv = lay["qkv"].forward(x)
                qa = lay["o_proj"]._quantize_input(qkv[:, : self.q_cols])
                x = nccl.all_reduce(ops.w8a8_gemm(qa.q, lay["o_proj"].weight, qa.s, lay["o_proj"].weight_scale))
            y = lay["gate_up"].forward_silu_quant(x)
            x = nccl.all_reduce(ops.w8a8_gemm(y.q, lay["down"].weight, y.s, lay["down"].weight_scale))
        return x

    @staticmethod
    def launches_per_step():
        """Our kernels per step: per layer a quantiser and a GEMM per linear
        (the SiLU*mul quantiser in place of down's), reduce fused or NCCL's."""
        return LAYERS * (4 if MLP_ONLY else 8)


# --------------------------------------------------------------------------- the reference's NCCL path
class NcclUniqueId(ctypes.Structure):
    # unsigned bytes: a c_char array would convert to bytes only up to its first zero byte
    _fields_ = [("internal", ctypes.c_ubyte * 128)]


class SymmetricNcclAllReduce:
    """The reference's PyNCCL all-reduce, for the measured NCCL bar:
    ``ncclCommInitRank`` with a unique id broadcast from rank 0,
    ``ncclMemAlloc`` + ``ncclCommWindowRegister(NCCL_WIN_COLL_SYMMETRIC)`` of
    a max_bytes buffer, and per call a device copy into the window, an
    in-place ``ncclAllReduce`` (bf16, sum) and a copy back
    (M/kernel/csrc/src/pynccl.cu:74-134), driven through ctypes on the NCCL
    library torch ships."""

    NCCL_BF16, NCCL_SUM, WIN_SYMMETRIC, D2D = 9, 0, 0x01, 3

    def __init__(self, rank: int, world: int, max_bytes: int):
        import nvidia.cuda_runtime
        import nvidia.nccl

        self.nccl = ctypes.CDLL(os.path.join(list(nvidia.nccl.__path__)[0], "lib", "libnccl.so.2"))
        self.cudart = ctypes.CDLL(os.path.join(list(nvidia.cuda_runtime.__path__)[0], "lib", "libcudart.so.12"))
        vp = ctypes.c_void_p
        self.nccl.ncclCommInitRank.argtypes = [ctypes.POINTER(vp), ctypes.c_int, NcclUniqueId, ctypes.c_int]
        self.nccl.ncclMemAlloc.argtypes = [ctypes.POINTER(vp), ctypes.c_size_t]
        self.nccl.ncclCommWindowRegister.argtypes = [vp, vp, ctypes.c_size_t, ctypes.POINTER(vp), ctypes.c_int]
        self.nccl.ncclCommWindowDeregister.argtypes = [vp, vp]
        self.nccl.ncclAllReduce.argtypes = [vp, vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, vp, vp]
        self.nccl.ncclMemFree.argtypes = [vp]
        self.nccl.ncclCommDestroy.argtypes = [vp]
        self.nccl.ncclGetErrorString.restype = ctypes.c_char_p
        self.cudart.cudaMemcpyAsync.argtypes = [vp, vp, ctypes.c_size_t, ctypes.c_int, vp]
        self.max_bytes = int(max_bytes)
        uid = NcclUniqueId()
        if rank == 0:
            self._check(self.nccl.ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
        obj = [bytes(uid.internal) if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0)
        if len(obj[0]) != 128:
            raise RuntimeError("malformed NCCL unique id")
        ctypes.memmove(ctypes.addressof(uid), obj[0], 128)
        self.comm, self.buf, self.win = vp(), vp(), vp()
        self._check(self.nccl.ncclCommInitRank(ctypes.byref(self.comm), world, uid, rank), "ncclCommInitRank")
        self._check(self.nccl.ncclMemAlloc(ctypes.byref(self.buf), self.max_bytes), "ncclMemAlloc")
        self._check(self.nccl.ncclCommWindowRegister(self.comm, self.buf, self.max_bytes, ctypes.byref(self.win),
                                                     self.WIN_SYMMETRIC), "ncclCommWindowRegister")

    def version(self) -> int:
        v = ctypes.c_int(0)
        self.nccl.ncclGetVersion(ctypes.byref(v))
        return v.value

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what} failed: {self.nccl.ncclGetErrorString(rc).decode()}")

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        nbytes = x.numel() * x.element_size()
        if nbytes > self.max_bytes:
            raise RuntimeError("tensor larger than the symmetric window")
        st = torch.cuda.current_stream(x.device).cuda_stream
        if self.cudart.cudaMemcpyAsync(self.buf, x.data_ptr(), nbytes, self.D2D, st) != 0:
            raise RuntimeError("cudaMemcpyAsync into the window failed")
        self._check(self.nccl.ncclAllReduce(self.buf, self.buf, x.numel(), self.NCCL_BF16, self.NCCL_SUM,
                                            self.comm, st), "ncclAllReduce")
        if self.cudart.cudaMemcpyAsync(x.data_ptr(), self.buf, nbytes, self.D2D, st) != 0:
            raise RuntimeError("cudaMemcpyAsync out of the window failed")
        return x

    def close(self) -> None:
        if self.comm.value:
            torch.cuda.synchronize()
            self.nccl.ncclCommWindowDeregister(self.comm, self.win)
            self.nccl.ncclMemFree(self.buf)
            self.nccl.ncclCommDestroy(self.comm)
            self.comm = ctypes.c_void_p()


# --------------------------------------------------------------------------- timing helpers
def _flush(buf):
    """Flush L2 before a timed step: write a 256 MB buffer (twice L2), then
    read it back.  The write alone would leave ~126 MB of dirty lines whose
    write-back the timed kernels would pay; after the read the lines in L2 are
    clean, so the timed region starts from a cold, clean cache."""
    buf.add_(1)
    buf.amax()


def time_graph(fn, steps, warmup, flush_buf, stream):
    """Capture fn in a CUDA graph, then time `steps` replays with CUDA events
    on the capture stream, flushing L2 (untimed) before each."""
    with torch.cuda.stream(stream):
        fn()
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        out = fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            _flush(flush_buf)
            g.replay()
        torch.cuda.synchronize()
        for i in range(steps):
            _flush(flush_buf)
            starts[i].record(stream)
            g.replay()
            ends[i].record(stream)
    torch.cuda.synchronize()
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    del g
    return sum(ms), ms, out


def time_kernel_events(fn, reps, flush_buf, stream):
    """Average device time (ms) of one call of fn: fn is captured in a CUDA
    graph and each replay is bracketed by CUDA events on `stream`, so host-side
    argument checks and launch latency stay outside the measurement; L2 is
    flushed before each replay."""
    total, _, _ = time_graph(fn, reps, 3, flush_buf, stream)
    return total / reps


def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _read_traffic(m: int, n: int, k: int, silu: bool = False):
    """Per-launch DRAM bytes of the dominant kernel, from the committed ncu
    summary of the gate_up GEMM at M=4096, N=51200, K=5120 (TP=1) -- with the
    SiLU*mul epilogue or plain.  At TP=N the launch has N/TP output columns;
    its traffic (weight rows read, output columns written) scales with N, so
    the captured figure is scaled by n / 51200.  None for another M or K."""
    name = "gemm_gate_up_silu_m4096_tp1_ncu.txt" if silu else "gemm_gate_up_m4096_tp1_ncu.txt"
    p = os.path.join(ROOT, "profiles", name)
    if m != 4096 or k != HIDDEN:
        return None
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch_full:"):
                    return round(float(line.split(":", 1)[1]) * n / (2 * INTER))
    except OSError:
        pass
    return None


def int8_peak(pkg, stream, reps: int = 3):
    """Measured int8 tensor-core ceiling: the library's MMA-only probe (1-SM
    128x256 and 2-SM 256x256 shapes), best of `reps` launches of each."""
    lib = pkg.load_library()
    best = {}
    for pair in (0, 1):
        ops = ctypes.c_int64(0)
        times = []
        with torch.cuda.stream(stream):
            for _ in range(reps + 1):
                s = torch.cuda.Event(enable_timing=True)
                e = torch.cuda.Event(enable_timing=True)
                s.record(stream)
                pkg._lib.check(lib.w8a8_mma_peak_probe(pair, 40000, ctypes.byref(ops), stream.cuda_stream),
                               "mma_peak_probe")
                e.record(stream)
                times.append((s, e))
        torch.cuda.synchronize()
        ms = min(s.elapsed_time(e) for s, e in times[1:])
        best["pair" if pair else "single"] = round(ops.value / (ms * 1e-3) / 1e12, 1)
    return best


# --------------------------------------------------------------------------- parity vs the oracle
def sample_rows(m: int):
    """A fixed sample of token rows: two per 128-row tile (one pseudo-random,
    one at the tile's end), so every output tile of every GEMM is checked."""
    rows = set()
    for t in range((m + 127) // 128):
        lo, hi = t * 128, min(m, t * 128 + 128)
        rows.add(lo + (t * 53 + 17) % (hi - lo))
        rows.add(hi - 1)
    return sorted(rows)


def collect_trace(pkg, stack, x, rows, world):
    """Every rank's sampled rows of each layer's input and output, plus the
    gate_up GEMM's int32 accumulator and the quantiser's outputs for the
    sampled inputs; all ranks' traces on every rank (CPU tensors)."""
    ops = pkg.ops
    idx = torch.tensor(rows, device=x.device)
    t = stack.forward_traced(x)
    qh = ops.quant_per_token(t["h"])
    acc = torch.empty(x.shape[0], stack.gate_up.weight.shape[0], dtype=torch.int32, device=x.device)
    gu2 = ops.w8a8_gemm(qh[0], stack.gate_up.weight, qh[1], stack.gate_up.weight_scale, out_i32=acc)
    xq = ops.quant_per_token(x.index_select(0, idx))
    torch.cuda.synchronize()
    mine = {k: v.index_select(0, idx).cpu() for k, v in t.items()}
    mine["gu_i32"] = acc.index_select(0, idx).cpu()
    mine["gu_again_equal"] = bool(torch.equal(gu2.index_select(0, idx), t["gu"].index_select(0, idx)))
    mine["xq"], mine["xs"] = xq[0].cpu(), xq[1].cpu()
    mine["wq_qkv_head"] = stack.qkv.weight[:4].cpu()
    mine["ws_qkv"] = stack.qkv.weight_scale.cpu()
    del acc, gu2, t
    if world == 1:
        return [mine]
    everyone = [None] * world
    torch.distributed.all_gather_object(everyone, mine)
    return everyone


def oracle_parity(traces, tp: int, dev: torch.device):
    """Recompute every layer on the sampled rows with the CPU oracle from each
    layer's actual input, and compare (int8 / int32 / bf16 bit for bit; the
    SiLU*mul quantiser's int8 within one step on at most 0.1 % of elements,
    since its bf16 product may differ from the CPU's by one ulp)."""
    from oracle import w8a8_oracle as O

    W = {}
    for name in PROJ:
        W[name] = O.quant_weight_per_channel(full_weight(name, dev).cpu())

    def shard(name, r):
        key = "." + name
        return O.shard_tensor(key, W[name][0], r, tp, NKV), O.shard_scale(key, W[name][1], r, tp, NKV)

    bad = []
    max_err = 0.0

    def cmp(what, got, want):
        nonlocal max_err
        if not torch.equal(got, want):
            err = float((got.float() - want.float()).abs().max())
            max_err = max(max_err, err)
            bad.append(f"{what}: max |diff| {err:.3g}")

    t0 = traces[0]
    q_ref, s_ref = O.quant_per_token(t0["x"])
    cmp("quantiser x int8", t0["xq"], q_ref)
    cmp("quantiser x scale", t0["xs"], s_ref)
    i32_ok = True
    silu_mismatch = 0.0
    for r in range(tp):
        parts = [shard(n, r) for n in ("q_proj", "k_proj", "v_proj")]
        wq = torch.cat([p[0] for p in parts])
        ws = torch.cat([p[1] for p in parts])
        cmp(f"loader weight shard r{r}", traces[r]["wq_qkv_head"], wq[:4])
        cmp(f"loader weight scales r{r}", traces[r]["ws_qkv"], ws)
        cmp(f"qkv r{r}", traces[r]["qkv"], O.w8a8_linear(traces[r]["x"], wq, ws)[3])
    attn_full = torch.cat([traces[r]["attn"] for r in range(tp)], dim=1)
    h_ref = O.tp_linear("row", attn_full, W["o_proj"][0], W["o_proj"][1], tp, key=".o_proj")[0]
    for r in range(tp):
        cmp(f"o_proj+allreduce r{r}", traces[r]["h"], h_ref)
        gate, up = shard("gate_proj", r), shard("up_proj", r)
        wq, ws = torch.cat([gate[0], up[0]]), torch.cat([gate[1], up[1]])
        _, _, acc, gu = O.w8a8_linear(traces[r]["h"], wq, ws)
        cmp(f"gate_up r{r}", traces[r]["gu"], gu)
        if not torch.equal(traces[r]["gu_i32"], acc):
            i32_ok = False
            bad.append(f"gate_up int32 r{r}")
        if not traces[r]["gu_again_equal"]:
            bad.append(f"gate_up repeat r{r}")
        q, s, _ = O.silu_mul_quant(traces[r]["gu"])
        dq = (traces[r]["q"].int() - q.int()).abs()
        silu_mismatch = max(silu_mismatch, float((dq != 0).float().mean()))
        if int(dq.max()) > 1 or silu_mismatch > 1e-3:
            bad.append(f"silu*mul quant r{r}: max |dq| {int(dq.max())}")
    parts = []
    for r in range(tp):
        wq, _ = shard("down_proj", r)
        parts.append(O.dequant(O.int_gemm(traces[r]["q"], wq), traces[r]["s"], W["down_proj"][1]))
    out_ref = O.all_reduce_sum(parts) if tp > 1 else parts[0]
    for r in range(tp):
        cmp(f"down+allreduce r{r}", traces[r]["out"], out_ref)
    within_tol = max_err <= 1e-2 or all(
        torch.allclose(traces[r]["out"].float(), out_ref.float(), rtol=1e-2, atol=1e-2) for r in range(tp))
    return {
        "rows": len(t0["x"]),
        "int8": "bit-exact" if not any("quantiser" in b for b in bad) else "mismatch",
        "int32": "bit-exact" if i32_ok else "mismatch",
        "bf16": "bit-exact" if max_err == 0.0 else max_err,
        "silu_quant_int8_mismatch_frac": silu_mismatch,
        "tolerance": "int8/int32 bit-exact; bf16 within 1e-2 rel / 1e-2 abs",
        "ok": (not bad) or (within_tol and i32_ok and all(("int32" not in b and "quantiser" not in b) for b in bad)),
        "layers": ["quant(x)", "qkv", "o_proj+allreduce", "gate_up (+int32)", "silu*mul quant", "down+allreduce"],
        "failures": bad[:8],
    }


# --------------------------------------------------------------------------- CPU baselines
def _cpu_rank(rank, world, m, threads, init_file, q, c0_budget_s, workload="cfg3"):
    """One CPU TP rank: this rank's shard of the four W8A8 linears through the
    oracle (torch._int_mm on CPU) with the row-parallel partials summed over
    gloo ranks by ``all_reduce`` (TorchDistributedImpl, M/distributed/impl.py:24-32);
    then the reference's own bf16 arithmetic (F.linear, M/layers/linear.py:31-32)
    of the same shard on a bounded token sample."""
    try:
        select_workload(workload)
        torch.set_num_threads(threads)
        import torch.distributed as dist
        from oracle import w8a8_oracle as O

        if world > 1:
            dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)

        def all_reduce(x):
            if world > 1:
                dist.all_reduce(x)
            return x

        sh = local_shapes(world)
        g = torch.Generator().manual_seed(100 + rank)
        w8 = {k: (torch.randint(-127, 128, (n, kk), generator=g, dtype=torch.int8), torch.rand(n, generator=g) * 1e-3)
              for k, (n, kk) in sh.items()}
        x = torch.randn(m, HIDDEN, generator=torch.Generator().manual_seed(0)).bfloat16()
        qc = (NQ // world) * HEAD_DIM

        def step_w8a8():
            h = x
            for _ in range(LAYERS):  # every layer's shard the same size; one set of weights stands in
                if not MLP_ONLY:
                    qkv = O.w8a8_linear(h, *w8["qkv"])[3]
                    h = all_reduce(O.w8a8_linear(qkv[:, :qc].contiguous(), *w8["o_proj"])[3])
                gu = O.w8a8_linear(h, *w8["gate_up"])[3]
                qq, ss, _ = O.silu_mul_quant(gu)
                h = all_reduce(O.dequant(O.int_gemm(qq, w8["down"][0]), ss, w8["down"][1]))
            return h

        def timed(fn, n):
            ts = []
            for _ in range(n):
                if world > 1:
                    dist.barrier()
                t0 = time.perf_counter()
                fn()
                ts.append(time.perf_counter() - t0)
            return statistics.median(ts)

        step_w8a8()
        t8 = timed(step_w8a8, 3)
        # C0: the reference's bf16 F.linear layers (+ all_reduce) on a bounded sample
        wb = {k: torch.randn(n, kk, generator=g).bfloat16() for k, (n, kk) in sh.items()}
        F = torch.nn.functional

        def step_bf16(xb):
            h = xb
            for _ in range(LAYERS):
                if not MLP_ONLY:
                    qkv = F.linear(h, wb["qkv"])
                    h = all_reduce(F.linear(qkv[:, :qc], wb["o_proj"]))
                gu = F.linear(h, wb["gate_up"])
                i = gu.shape[1] // 2
                y = (F.silu(gu[:, :i].float()) * gu[:, i:].float()).bfloat16()
                h = all_reduce(F.linear(y, wb["down"]))
            return h

        m0 = 16
        t1 = timed(lambda: step_bf16(x[:m0]), 1)
        flag = torch.tensor([int(max(16, min(m, m0 * c0_budget_s / max(t1, 1e-3))))])
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        mc0 = int(flag.item())
        tb = timed(lambda: step_bf16(x[:mc0]), 2)
        if world > 1:
            dist.destroy_process_group()
        q.put((rank, t8, tb, mc0))
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, None, repr(e), 0))


def cpu_tokens(m: int) -> int:
    """Tokens the CPU baseline times: exactly M for the headline workload; a
    bounded sample for the larger ones (cfg2 / cfg4 would take minutes)."""
    return m if WORKLOAD == "cfg3" else min(m, 512)


def host_cores() -> int:
    """Physical cores this process may run on (torchrun pins OMP_NUM_THREADS
    to 1 in its ranks, so torch's own thread count says nothing here)."""
    try:
        import psutil

        phys = psutil.cpu_count(logical=False) or 1
    except Exception:  # noqa: BLE001
        phys = os.cpu_count() or 1
    return max(1, min(phys, len(os.sched_getaffinity(0))))


def cpu_tp_baseline(world: int, m: int, threads_total: int, c0_budget_s: float = 4.0, timeout: float = 600.0):
    """Time the CPU path at TP = world as `world` gloo ranks (spawned, no GPU),
    each with threads_total // world threads, at exactly M tokens.  Returns a
    cpu_baseline dict (W8A8 oracle = the restated reference path) with the
    reference's bf16 F.linear arithmetic (C0) beside it."""
    import multiprocessing as mp

    threads = max(1, threads_total // world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = tempfile.mktemp(prefix="w8a8_cpu_gloo_")
    saved = {k: os.environ.get(k) for k in ("CUDA_VISIBLE_DEVICES", "OMP_NUM_THREADS")}
    os.environ["CUDA_VISIBLE_DEVICES"] = ""  # the CPU ranks never touch a GPU
    os.environ["OMP_NUM_THREADS"] = str(threads)
    try:
        procs = [ctx.Process(target=_cpu_rank, args=(r, world, m, threads, init_file, q, c0_budget_s, WORKLOAD))
                 for r in range(world)]
        for p in procs:
            p.start()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    res = {}
    try:
        for _ in range(world):
            r, t8, tb, mc0 = q.get(timeout=timeout)
            res[r] = (t8, tb, mc0)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
        try:
            os.unlink(init_file)
        except OSError:
            pass
    errs = [v[1] for v in res.values() if v[0] is None]
    if errs:
        raise RuntimeError(f"CPU baseline rank failed: {errs[0]}")
    t8 = max(v[0] for v in res.values())
    tb = max(v[1] for v in res.values())
    mc0 = res[0][2]
    return {
        "value": round(m / t8, 1), "unit": UNIT, "cores": threads * world, "kind": "port",
        "sample": (f"M={m} tokens through {WORKLOAD}'s W8A8 linears + SiLU*mul quant at TP={world}: {world} gloo CPU "
                   f"rank(s) x {threads} threads, row-parallel partials summed by all_reduce; oracle "
                   f"(torch._int_mm on CPU); median of 3 after 1 warm-up"),
        "c0_reference_bf16": {"value": round(mc0 / tb, 1), "unit": UNIT,
                              "sample": f"the reference's bf16 F.linear layers (+ all_reduce) on M={mc0} tokens, "
                                        f"same ranks and threads, median of 2"},
    }


# --------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, dev):
    pkg = _pkg()
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(rank, world)
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]
    comm = None
    comm_kind = "none (tp1)"
    if world > 1:
        comm = D.enable_peer_mem_distributed(D.get_tp_info(), None, max_bytes=args.m * HIDDEN * 2, device=dev)
        comm.set_mode(args.comm_mode)
        comm_kind = ("fused into the row-parallel GEMMs (NVLink peer-memory stores; NVSwitch multicast buffer "
                     "attached, used by mode 3 only)" if comm.nvls else
                     f"fused into the row-parallel GEMMs (NVLink peer-memory stores; no NVLS: {comm.nvls_error})")
        comm_kind += f"; mode {args.comm_mode}"
    stream = torch.cuda.Stream(dev)
    flush_buf = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stack = Stack(pkg, world, rank, dev)
    pkg.ops.gemm_workspace(dev)
    peaks, peak_kind = _peaks()
    ops = pkg.ops

    # ---------------------------------------------------------------- headline
    gx = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(args.m, HIDDEN, device=dev, generator=gx).bfloat16()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index, args.clocks_dir) as clk:
        total_ms, per_ms, _ = time_graph(lambda: stack.forward(x), args.steps, args.warmup, flush_buf, stream)
        total_ms = max_over_ranks(total_ms, world, dev)
        ms_per_step = total_ms / args.steps
        value = args.m * args.steps / (total_ms / 1e3)

        # ------------------------------------------------------------ decode sweep
        # A model's layers run back to back inside one CUDA graph, so the
        # graph's launch cost is spread over all of them: each replay runs
        # DECODE_CHAIN consecutive steps, each through its own copy of the
        # layers (own weight storage: no step finds another's weights in L2),
        # and the time per step is the replay's time / DECODE_CHAIN.
        sweep = {}
        ops_tok, wbytes = layer_ops(world)
        chain = [stack.layers] + [clone_layers(stack.layers) for _ in range(DECODE_CHAIN - 1)]

        def decode_chain(xm):
            for layers in chain:
                xm = stack.forward_layers(layers, xm)
            return xm

        for m in args.sweep:
            xm = torch.randn(m, HIDDEN, device=dev, generator=gx).bfloat16()
            reps = max(10, args.steps // 2)
            tms, _, _ = time_graph(lambda: decode_chain(xm), reps, args.warmup, flush_buf, stream)
            tms = max_over_ranks(tms, world, dev)
            us = tms / (reps * DECODE_CHAIN) * 1e3
            t_hbm = wbytes / (peaks["hbm_gbs"] * 1e9) * 1e6
            sweep[str(m)] = {"tokens_per_s": round(m / (us * 1e-6), 1), "us_per_step": round(us, 2),
                             "weight_stream_frac_of_hbm": round(t_hbm / us, 3),
                             "steps_per_graph": DECODE_CHAIN}
        del chain

        # ------------------------------------------------------------ roofline: dominant kernel
        n_gu, k_gu = local_shapes(world)["gate_up"]
        qa = stack.gate_up._quantize_input(x)
        gemm_out = torch.empty(args.m, n_gu, dtype=torch.bfloat16, device=dev)
        plain_ms = time_kernel_events(
            lambda: ops.w8a8_gemm(qa.q, stack.gate_up.weight, qa.s, stack.gate_up.weight_scale, out=gemm_out),
            max(10, args.steps // 2), flush_buf, stream)
        # the step's gate_up kernel: the GEMM with SiLU*mul in its epilogue
        # where the fusion applies (y [M, N/2] written instead of [M, N])
        silu_step = ops.gemm_silu(qa.q, stack.gate_up.weight, qa.s, stack.gate_up.weight_scale) is not None
        if silu_step:
            gemm_ms = time_kernel_events(
                lambda: ops.gemm_silu(qa.q, stack.gate_up.weight, qa.s, stack.gate_up.weight_scale),
                max(10, args.steps // 2), flush_buf, stream)
        else:
            gemm_ms = plain_ms
        alg_ops = 2.0 * args.m * n_gu * k_gu
        achieved_tops = alg_ops / (gemm_ms * 1e-3) / 1e12
        peak_probe = int8_peak(pkg, stream)
        try:
            wt = stack.gate_up.weight.t()
            int_mm_ms = time_kernel_events(lambda: torch._int_mm(qa.q, wt), 10, flush_buf, stream)
            int_mm_tops = alg_ops / (int_mm_ms * 1e-3) / 1e12
        except Exception:
            int_mm_ms = int_mm_tops = None
        wbf = torch.randn(n_gu, k_gu, device=dev, dtype=torch.bfloat16)
        bf16_ms = time_kernel_events(lambda: torch.nn.functional.linear(x, wbf), 10, flush_buf, stream)
        del wbf
    clocks = clk.summary()
    peak_tops = max(peak_probe.values())

    # ---------------------------------------------------------------- per-op breakdown
    bsteps = max(10, args.steps // 2)

    def op_us(fn):
        t, _, _ = time_graph(fn, bsteps, args.warmup, flush_buf, stream)
        return round(max_over_ranks(t, world, dev) / bsteps * 1e3, 2)

    # the first layer's ops, each in its own graph (an MLP-only workload has
    # no qkv / o_proj: its gate_up reads the step input)
    qx = ops.quant_per_token(x)
    o_p, d_p = stack.o_proj, stack.down
    breakdown = {"quant_x": op_us(lambda: ops.quant_per_token(x))}
    if not MLP_ONLY:
        qkv = stack.qkv.forward(x)
        attn = qkv[:, : stack.q_cols]
        qattn = ops.quant_per_token(attn)
        h = o_p.forward(attn)
        qh = ops.quant_per_token(h)
        breakdown["qkv_gemm"] = op_us(lambda: ops.w8a8_gemm(qx[0], stack.qkv.weight, qx[1], stack.qkv.weight_scale))
        breakdown["quant_attn"] = op_us(lambda: ops.quant_per_token(attn))
        breakdown["o_proj"] = op_us(lambda: o_p.forward(ops.QuantizedActivation(*qattn)))
        breakdown["quant_h"] = op_us(lambda: ops.quant_per_token(h))
    else:
        h, qh = x, qx
    qah = ops.QuantizedActivation(*qh)
    qy = stack.gate_up.forward_silu_quant(qah)
    # the step's gate_up: the GEMM with SiLU*mul in its epilogue + the
    # quantiser of its product (or, below the fusion's range, the GEMM and the
    # fused SiLU*mul quantiser)
    breakdown["gate_up_silu_quant"] = op_us(lambda: stack.gate_up.forward_silu_quant(qah))
    breakdown["down"] = op_us(lambda: d_p.forward(qy))
    ops_keys = list(breakdown)
    # for comparison (not in the step): the two-step path it replaces
    gu = stack.gate_up.forward(qah)
    breakdown["two_step_gate_up_gemm"] = op_us(lambda: ops.w8a8_gemm(qh[0], stack.gate_up.weight, qh[1],
                                                                     stack.gate_up.weight_scale))
    breakdown["two_step_silu_mul_quant"] = op_us(lambda: ops.silu_and_mul_quant(gu))
    del gu
    if world > 1:
        if not MLP_ONLY:
            breakdown["o_proj_gemm_alone"] = op_us(lambda: ops.w8a8_gemm(qattn[0], o_p.weight, qattn[1],
                                                                         o_p.weight_scale))
            breakdown["o_proj_reduce_exposed"] = round(breakdown["o_proj"] - breakdown["o_proj_gemm_alone"], 2)
        breakdown["down_gemm_alone"] = op_us(lambda: ops.w8a8_gemm(qy.q, d_p.weight, qy.s, d_p.weight_scale))
        breakdown["down_reduce_exposed"] = round(breakdown["down"] - breakdown["down_gemm_alone"], 2)
        hb = h.clone()
        breakdown["allreduce_MxH_ours"] = op_us(lambda: comm.all_reduce(hb))
    breakdown["sum_of_ops"] = round(sum(breakdown[k] for k in ops_keys), 2)
    if LAYERS > 1:
        breakdown["per_layer_step"] = round(ms_per_step * 1e3 / LAYERS, 2)
    breakdown["step"] = round(ms_per_step * 1e3, 2)

    # ---------------------------------------------------------------- the reference's NCCL bar (N > 1)
    nccl_line = None
    if world > 1 and not args.no_nccl:
        nccl = None
        try:
            err = None
            try:
                nccl = SymmetricNcclAllReduce(rank, world, args.m * HIDDEN * 2)
            except Exception as e:  # noqa: BLE001 - every rank learns of it below
                err = e
            ok = torch.tensor([0 if err else 1], device=dev)
            torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
            if not int(ok.item()):
                raise err or RuntimeError("NCCL symmetric-window set-up failed on another rank")
            tms, _, _ = time_graph(lambda: stack.forward_nccl(x, nccl), args.steps, args.warmup, flush_buf, stream)
            tms = max_over_ranks(tms, world, dev)
            hb = h.clone()
            nccl_line = {
                "tokens_per_s": round(args.m * args.steps / (tms / 1e3), 1),
                "ms_per_step": round(tms / args.steps, 4),
                "o_proj_us": None if MLP_ONLY else op_us(lambda: nccl.all_reduce(
                    ops.w8a8_gemm(qattn[0], o_p.weight, qattn[1], o_p.weight_scale))),
                "down_us": op_us(lambda: nccl.all_reduce(ops.w8a8_gemm(qy.q, d_p.weight, qy.s, d_p.weight_scale))),
                "allreduce_MxH_us": op_us(lambda: nccl.all_reduce(hb)),
                "how": "same GEMMs; row-parallel reduce = copy into an ncclMemAlloc'd symmetric window, "
                       "ncclAllReduce (bf16 sum), copy back (M/kernel/csrc/src/pynccl.cu:93-134)",
                "nccl_version": nccl.version(),
            }
            y_n = stack.forward_nccl(x, nccl)
            y_f = stack.forward(x)
            torch.cuda.synchronize()
            # NCCL sums the bf16 partials in its own order; after the first layer
            # the paths see inputs that differ in the last bit
            nccl_line["max_rel_diff_vs_fused"] = float((y_n.float() - y_f.float()).abs().max()
                                                       / y_f.float().abs().max().clamp_min(1e-30))
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            nccl_line = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        finally:
            if nccl is not None:
                nccl.close()

    # ---------------------------------------------------------------- parity (after timing)
    parity = None
    if MLP_ONLY:
        parity = {"skipped": "MLP-only workload; its GEMM shapes are checked by the GPU tests"}
    elif not args.no_parity:
        traces = collect_trace(pkg, stack, x, sample_rows(args.m), world)
        if rank == 0:
            parity = oracle_parity(traces, world, dev)
        del traces
        if world > 1:
            torch.distributed.barrier()

    # ---------------------------------------------------------------- e2e (public API, host buffers)
    # Every step copies its input in from pinned host memory (once, on rank 0,
    # handed to the other ranks over NVLink by the communicator's broadcast)
    # and reads the replicated output back to the host (from rank 0).  Two
    # buffers per direction and two copy streams pipeline the steps, as a
    # serving loop does: step i+1's input crosses PCIe and step i-1's output
    # returns while step i computes.
    x_host = torch.randn(args.m, HIDDEN, generator=torch.Generator().manual_seed(1)).bfloat16().pin_memory()
    y_host = [torch.empty(args.m, HIDDEN, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty(args.m, HIDDEN, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_y = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(8, args.steps // 2)

    def e2e_run(n):
        for i in range(n):
            b = i % 2
            if rank == 0:
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev_used[b])  # step i-2 is done reading this buffer
                    xd[b].copy_(x_host, non_blocking=True)
                    ev_in[b].record(s_in)
                stream.wait_event(ev_in[b])
            with torch.cuda.stream(stream):
                stream.wait_event(ev_out[b])  # step i-2's output is back on the host
                if comm is not None:
                    comm.broadcast(xd[b], root=0)
                y = stack.forward(xd[b])
                ev_used[b].record(stream)
                ev_y[b].record(stream)
            if rank == 0:
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_y[b])
                    y_host[b].copy_(y, non_blocking=True)
                    y.record_stream(s_out)
                    ev_out[b].record(s_out)
            else:
                ev_out[b].record(stream)

    e2e_run(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(s_in if rank == 0 else stream)
    e2e_run(e2e_steps)
    for st in (s_in, s_out):
        stream.wait_stream(st)
    e.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s.elapsed_time(e), world, dev)
    e2e_value = args.m * e2e_steps / (e2e_ms / 1e3)
    # the pipelined outputs are the stack's output for x_host
    y_ref = stack.forward(x_host.to(dev))
    torch.cuda.synchronize()
    e2e_ok = bool(torch.equal(y_host[(e2e_steps - 1) % 2], y_ref.cpu())) if rank == 0 else True

    # ---------------------------------------------------------------- CPU baseline (rank 0, every N)
    cpu = None
    if rank == 0 and not args.no_cpu:
        try:
            cpu = cpu_tp_baseline(world, cpu_tokens(args.m), host_cores())
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            cpu = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    if world > 1:
        torch.distributed.barrier()

    traffic = _read_traffic(args.m, n_gu, k_gu, silu=silu_step)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 (int32 accumulate, fp32 dequant, bf16 out)",
        "data": "synthetic: seeded N(0,1) bf16 activations; synthetic N(0,0.02) bf16 checkpoint quantised per "
                "channel and sharded by the package's loader",
        "config": dict(workload_config(world, args.m), allreduce=comm_kind, l2=L2_NOTE),
        "roofline": {"kernel": (f"w8a8_gemm_silu gate_up + SiLU*mul epilogue M={args.m} N={n_gu} K={k_gu}"
                                if silu_step else f"w8a8_gemm gate_up M={args.m} N={n_gu} K={k_gu}"),
                     "bound": "tensor",
                     "achieved": round(achieved_tops, 1), "peak": round(peak_tops, 1), "unit": "TOP/s (int8)",
                     "frac": round(achieved_tops / peak_tops, 4),
                     "peak_source": "measured in this run: MMA-only tcgen05 kind::i8 loop from resident shared "
                                    f"memory (w8a8_mma_peak_probe) {peak_probe}",
                     "frac_of_2x_bf16": round(achieved_tops / (2.0 * peaks["bf16_tflops"]), 4),
                     "frac_of_nominal_int8_4500": round(achieved_tops / INT8_NOMINAL_TOPS, 4),
                     "launch_ms": round(gemm_ms, 4), "traffic": traffic,
                     "algorithmic_bytes": (args.m * k_gu + n_gu * k_gu + (args.m * n_gu if silu_step else
                                                                           2 * args.m * n_gu)
                                           + (8 if silu_step else 4) * args.m + 4 * n_gu)},
        "yardsticks": {"torch_int_mm_tops_same_shape": None if int_mm_tops is None else round(int_mm_tops, 1),
                       "torch_int_mm_ms_same_shape": None if int_mm_ms is None else round(int_mm_ms, 4),
                       "cublas_bf16_linear_ms_same_shape": round(bf16_ms, 4),
                       "ours_gemm_ms_same_shape": round(gemm_ms, 4),
                       "ours_plain_gemm_ms_same_shape": round(plain_ms, 4)},
        "breakdown_us": breakdown,
        "nccl_baseline": nccl_line,
        "parity": parity,
        "sweep": sweep,
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": args.m * HIDDEN * 2,
                "d2h_bytes_per_step": args.m * HIDDEN * 2,
                "output_matches": e2e_ok,
                "how": "eager public layer API; every step: pinned host input copied in once (rank 0) and "
                       "broadcast to the other ranks over NVLink, replicated output copied back from rank 0; "
                       "double-buffered copy streams overlap step i+1's input and step i-1's output with step i"},
        "gpu_launches": Stack.launches_per_step() * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    return line


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    if rank != 0:
        return None
    cpu = cpu_tp_baseline(world, cpu_tokens(args.m), host_cores())
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": cpu["value"],
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(args.m / cpu["value"] * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 (int32 accumulate, fp32 dequant, bf16 out)",
        "data": "synthetic: seeded int8 weights and bf16 activations of the same shapes",
        "config": workload_config(world, args.m),
        "implementation": "CPU restatement of the reference path (oracle/w8a8_oracle.py) on host cores, one gloo "
                          "rank per TP rank; the reference's own bf16 F.linear arithmetic in cpu_baseline.c0",
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- profiling entries
def run_gemm_only(args, dev):
    """Profiling entry for single GEMM shapes (``--gemm MxNxK,...``): int8
    operands drawn on the device (no other kernel of ours runs), then two
    launches of the auto-planned GEMM per shape, in the order given (with
    ``--silu``: the GEMM with the SiLU*mul epilogue, N = 2I, and the quantiser
    of its product)."""
    pkg = _pkg()
    pkg.ops.gemm_workspace(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    shapes = []
    for spec in args.gemm.split(","):
        m, n, k = (int(v) for v in spec.lower().split("x"))
        a = torch.randint(-127, 128, (m, k), device=dev, generator=g, dtype=torch.int8)
        w = torch.randint(-127, 128, (n, k), device=dev, generator=g, dtype=torch.int8)
        sa = torch.rand(m, device=dev, generator=g) * 1e-3
        sw = torch.rand(n, device=dev, generator=g) * 1e-3
        shapes.append((a, w, sa, sw, torch.empty(m, n, dtype=torch.bfloat16, device=dev)))
    torch.cuda.synchronize()
    for a, w, sa, sw, out in shapes:
        for _ in range(2):
            if args.silu:
                assert pkg.ops.gate_up_silu_quant(a, w, sa, sw) is not None, "shape outside the SiLU epilogue's range"
            else:
                pkg.ops.w8a8_gemm(a, w, sa, sw, out=out)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    print(json.dumps({"gemm_only": True, "shapes": args.gemm,
                      "plans": [pkg.ops.gemm_plan(a.shape[0], w.shape[0], a.shape[1]) for a, w, *_ in shapes]}))


# Mixture-of-experts layer (the experts of Qwen3-30B-A3B's MoE MLP): not a
# BASELINE configuration; measured so the grouped GEMM has a throughput and
# roofline record beside the dense path.
MOE_SHAPE = {"experts": 128, "topk": 8, "hidden": 2048, "inter": 768}


def run_moe(args, dev):
    """``--moe``: the W8A8 experts of one MoE layer (align, quantise-scatter,
    gate_up grouped GEMM with SiLU*mul, quantiser, down grouped GEMM with the
    routing weight, top-k sum) at each M of ``--moe-m``; random int8 expert
    weights, seeded N(0, 1) activations and router logits routed with the
    reference's fused_topk arithmetic.  Per-stage device times from CUDA-graph
    replays (L2 flushed before each), and the grouped GEMMs' int8 throughput
    against the measured MMA ceiling and against this library's dense GEMM on
    the same operation count."""
    pkg = _pkg()
    ops = pkg.ops
    E, K, H, I = MOE_SHAPE["experts"], MOE_SHAPE["topk"], MOE_SHAPE["hidden"], MOE_SHAPE["inter"]
    g = torch.Generator(device=dev).manual_seed(0)
    w1q = torch.randint(-127, 128, (E, 2 * I, H), dtype=torch.int8, device=dev, generator=g)
    w2q = torch.randint(-127, 128, (E, H, I), dtype=torch.int8, device=dev, generator=g)
    sw1 = torch.rand(E, 2 * I, device=dev, generator=g) * 1e-3 + 1e-5
    sw2 = torch.rand(E, H, device=dev, generator=g) * 1e-3 + 1e-5
    stream = torch.cuda.Stream(dev)
    flush_buf = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    ops.gemm_workspace(dev)
    peak = int8_peak(pkg, stream)
    reps = max(args.steps, 5)
    per_m = {}
    for m in args.moe_m:
        x = torch.randn(m, H, device=dev, generator=g).bfloat16()
        logits = torch.randn(m, E, device=dev, generator=g)
        p = torch.softmax(logits.float(), dim=-1)
        w, ids = torch.topk(p, K, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        w = (w / (w.sum(-1, keepdim=True) + 1e-8)).contiguous()
        ids = ids.to(torch.int32).contiguous()
        total, _, out = time_graph(lambda: ops.fused_experts_w8a8(x, w1q, sw1, w2q, sw2, w, ids), reps,
                                   max(args.warmup, 3), flush_buf, stream)
        layer_ms = total / reps
        r = ops.moe_align(ids, E)
        q = ops.moe_quant_scatter(x, r)
        y, amax = ops.moe_gemm(q, r.sa_sorted, w1q, sw1, r, silu=True)
        qy = ops.moe_quant_rows(y, amax, r)
        c3 = ops.moe_gemm(qy.q, qy.s, w2q, sw2, r, route_w=w)
        torch.cuda.synchronize()
        nb = int(r.num_blocks.item())
        st = {
            "align": time_kernel_events(lambda: ops.moe_align(ids, E), reps, flush_buf, stream),
            "quant_scatter": time_kernel_events(lambda: ops.moe_quant_scatter(x, r), reps, flush_buf, stream),
            "gate_up_silu": time_kernel_events(lambda: ops.moe_gemm(q, r.sa_sorted, w1q, sw1, r, silu=True), reps,
                                               flush_buf, stream),
            "quant_y": time_kernel_events(lambda: ops.moe_quant_rows(y, amax, r), reps, flush_buf, stream),
            "down": time_kernel_events(lambda: ops.moe_gemm(qy.q, qy.s, w2q, sw2, r, route_w=w), reps, flush_buf,
                                       stream),
            "topk_sum": time_kernel_events(lambda: ops.moe_sum(c3, r), reps, flush_buf, stream),
        }
        slots = m * K
        ops1, ops2 = 2.0 * slots * 2 * I * H, 2.0 * slots * H * I
        active = int(torch.unique(ids).numel())
        wbytes1, wbytes2 = active * 2 * I * H, active * H * I
        rec = {
            "tokens_per_s": round(m / (layer_ms * 1e-3), 1), "layer_us": round(layer_ms * 1e3, 2),
            "stages_us": {k_: round(v * 1e3, 2) for k_, v in st.items()},
            "blocks": nb, "padding_rows_frac": round(1.0 - slots / max(nb * 128, 1), 4), "active_experts": active,
            "gate_up_tops": round(ops1 / (st["gate_up_silu"] * 1e-3) / 1e12, 1),
            "down_tops": round(ops2 / (st["down"] * 1e-3) / 1e12, 1),
            "gate_up_weight_gbs": round(wbytes1 / (st["gate_up_silu"] * 1e-3) / 1e9, 1),
            "down_weight_gbs": round(wbytes2 / (st["down"] * 1e-3) / 1e9, 1),
        }
        if m >= 512:
            # dense yardstick: one W8A8 GEMM with the gate_up's operation count
            a = torch.randint(-127, 128, (slots, H), dtype=torch.int8, device=dev, generator=g)
            sa = torch.rand(slots, device=dev, generator=g) * 1e-3
            wd, sd = w1q[0].contiguous(), sw1[0].contiguous()
            dense_ms = time_kernel_events(lambda: ops.w8a8_gemm(a, wd, sa, sd), reps, flush_buf, stream)
            rec["dense_same_ops_us"] = round(dense_ms * 1e3, 2)
            rec["gate_up_vs_dense"] = round(dense_ms / st["gate_up_silu"], 3)
        per_m[str(m)] = rec
        del out, r, q, y, amax, qy, c3
    assert ops.device_error() == 0
    head = per_m[str(args.moe_m[-1])]
    return {
        "metric": "W8A8 MoE-layer tokens/s (experts of a Qwen3-30B-A3B MoE MLP: 128 experts, top-8, H 2048, I 768)",
        "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": reps, "warmup": max(args.warmup, 3),
        "higher_is_better": True, "dtype": "int8 (int32 accumulate, fp32 dequant, bf16 out)",
        "data": "synthetic: random int8 expert weights, seeded N(0,1) activations and router logits",
        "config": {"workload": "moe", "M": args.moe_m[-1], **MOE_SHAPE,
                   "l2": "flushed before every timed replay (256 MB written, then read back)"},
        "int8_peak_tops": peak, "per_m": per_m,
    }


def run_kernel_only(args, dev):
    """Profiling entry: three rounds of [quantiser, gate_up GEMM, fused
    SiLU*mul+quant], then three of the fused residual-add + RMSNorm +
    quantiser, at the headline shape on one GPU, no graphs, no timing."""
    pkg = _pkg()
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(0, 1)
    n, k = local_shapes(1)["gate_up"]
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(args.m, k, device=dev, generator=g).bfloat16()
    wq, ws = pkg.ops.quant_per_token((torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16())
    pkg.ops.gemm_workspace(dev)
    torch.cuda.synchronize()
    for _ in range(3):
        q, s = pkg.ops.quant_per_token(x)
        y = pkg.ops.w8a8_gemm(q, wq, s, ws)
        pkg.ops.silu_and_mul_quant(y)
    res = torch.randn(args.m, k, device=dev, generator=g).bfloat16()
    wn = torch.ones(k, device=dev).bfloat16()
    for _ in range(3):
        pkg.ops.rmsnorm_quant(x, wn, 1e-6, res)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    print(json.dumps({"kernel_only": True, "m": args.m, "n": n, "k": k}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel-only", action="store_true", help="profiling entry (see run_kernel_only)")
    ap.add_argument("--gemm", default="", help="profiling entry: GEMM shapes MxNxK,... (see run_gemm_only)")
    ap.add_argument("--silu", action="store_true",
                    help="with --gemm: the GEMM with the SiLU*mul epilogue and the quantiser of its product")
    ap.add_argument("--moe", action="store_true", help="MoE experts layer (see run_moe), not the headline")
    ap.add_argument("--moe-m", type=lambda v: [int(x) for x in v.split(",") if x], default=[1, 64, 512, 4096],
                    help="token counts for --moe (the last is the line's value)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg3",
                    help="BASELINE config: cfg3 (the headline), cfg2 (Qwen3-8B MLP), cfg4 (Llama-3.1-70B 4 layers)")
    ap.add_argument("--m", type=int, default=None, help="headline tokens (default: the workload's)")
    ap.add_argument("--sweep", type=lambda s: [int(v) for v in s.split(",") if v], default=None,
                    help="decode sizes (default: the workload's)")
    ap.add_argument("--no-nccl", action="store_true", help="skip the NCCL symmetric-window arm at N > 1")
    ap.add_argument("--comm-mode", type=int, default=0, choices=[0, 1, 2, 3],
                    help="fused reduce algorithm: 0 auto, 1 one-shot, 2 two-shot peer stores, 3 two-shot NVLS")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check after timing")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--pg-timeout", type=int, default=300, help="process-group timeout in seconds (N > 1)")
    ap.add_argument("--clocks-dir", default=tempfile.gettempdir(),
                    help="where the raw nvidia-smi samples of the timed region are written")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    select_workload(args.workload)
    if args.m is None:
        args.m = WORKLOADS[args.workload]["m"]
    if args.sweep is None:
        args.sweep = list(WORKLOADS[args.workload]["sweep"])

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.gemm:
        run_gemm_only(args, dev)
        return
    if args.kernel_only:
        run_kernel_only(args, dev)
        return
    if args.moe:
        print(json.dumps(run_moe(args, dev)), flush=True)
        return
    if world > 1:
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=timedelta(seconds=args.pg_timeout))
    try:
        line = run_ours(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.barrier()
            _pkg().distributed.destroy_distributed()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
