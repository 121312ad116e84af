"""Benchmark of the W8A8 tensor-parallel linear path on B200.

Workload: the four quantised linears of one Qwen3-32B
decoder layer at TP = N — qkv (column-parallel) -> o_proj (row-parallel +
all-reduce) -> gate_up (column-parallel) -> fused SiLU*mul + per-token quant
-> down (row-parallel + all-reduce).  Attention is not part of the path: the
q slice of the qkv output stands in for the attention output that feeds
o_proj.  hidden 5120, 64 q / 8 kv heads x 128, intermediate 25600.  A step is
one pass of that stack over M tokens (headline M = 4096, the prefill chunk;
the decode sizes M = 1, 32, 128, 256 are reported in ``sweep``).  Synthetic
seeded data: activations ~N(0, 1) bf16, weights ~N(0, 0.02) bf16 quantised per
output channel by the library's own quantiser.

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 launch one rank per GPU with torchrun (RANK / WORLD_SIZE from env).
Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
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

HIDDEN, HEAD_DIM, NQ, NKV, INTER = 5120, 128, 64, 8, 25600
METRIC = "W8A8 TP-layer tokens/s (Qwen3-32B decoder-layer linears: qkv, o_proj+AR, gate_up, silu*mul+quant, down+AR)"
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20
INT8_NOMINAL_TOPS = 4500.0


def _pkg():
    return importlib.import_module("mini-sglang-fork_b200")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def local_shapes(tp: int):
    """Per-rank (N, K) of qkv, o_proj, gate_up, down (M/layers/linear.py:56-127)."""
    lq = NQ // tp
    lkv = max(1, NKV // tp)
    return {
        "qkv": ((lq + 2 * lkv) * HEAD_DIM, HIDDEN),
        "o_proj": (HIDDEN, NQ * HEAD_DIM // tp),
        "gate_up": (2 * INTER // tp, HIDDEN),
        "down": (HIDDEN, INTER // tp),
    }


def layer_ops(tp: int):
    """Integer ops (2*M*N*K summed) and weight bytes of the four linears per token."""
    sh = local_shapes(tp)
    ops_per_token = sum(2 * n * k for n, k in sh.values())
    wbytes = sum(n * k + 4 * n for n, k in sh.values())
    return ops_per_token, wbytes


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


# --------------------------------------------------------------------------- our arm
class Stack:
    """The four W8A8 layers of one decoder layer on this rank, built through
    the package's public layer classes and loaded with load_state_dict."""

    def __init__(self, pkg, tp: int, rank: int, dev: torch.device):
        L = pkg.layers
        self.pkg = pkg
        self.qkv = L.LinearQKVMerged(HIDDEN, HEAD_DIM, NQ, NKV, has_bias=False)
        self.o_proj = L.LinearOProj(NQ * HEAD_DIM, HIDDEN, has_bias=False)
        self.gate_up = L.LinearColParallelMerged(HIDDEN, [INTER, INTER], has_bias=False)
        self.down = L.LinearRowParallel(INTER, HIDDEN, has_bias=False)
        self.q_cols = (NQ // tp) * HEAD_DIM
        g = torch.Generator(device=dev).manual_seed(1000 + 8 * rank)
        for i, layer in enumerate((self.qkv, self.o_proj, self.gate_up, self.down)):
            n, k = layer.weight.shape
            w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
            wq, ws = pkg.ops.quant_per_token(w)  # per-output-channel = per-row rule
            del w
            layer.load_state_dict({"weight": wq, "weight_scale": ws})

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        qkv = self.qkv.forward(x)
        attn = qkv[:, : self.q_cols]
        h = self.o_proj.forward(attn)
        gu = self.gate_up.forward(h)
        y = self.pkg.ops.silu_and_mul_quant(gu)
        return self.down.forward(y)

    launches_per_step = 8  # 3 quantisers + 1 fused silu*mul+quant + 4 GEMMs (reduce fused or NCCL)


def _flush(buf):
    buf.add_(1)


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
    """Average device time of one launch of fn (CUDA events on `stream`)."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            _flush(flush_buf)
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            ts.append((s, e))
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in ts) / reps


def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _read_traffic(m: int, n: int, k: int):
    """Per-launch DRAM bytes of the dominant kernel, from the committed ncu
    summary of the gate_up GEMM at M=4096, N=51200, K=5120 (TP=1).  At TP=N
    the launch has N/TP output columns; its traffic (weight rows read, output
    columns written) scales with N, so the captured figure is scaled by
    n / 51200.  None for another M or K."""
    p = os.path.join(ROOT, "profiles", "gemm_gate_up_m4096_tp1_ncu.txt")
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


def cpu_oracle_sample(tp: int, budget_s: float = 15.0):
    """Time the CPU oracle (the restated reference path) on a bounded sample of
    the same workload: all TP ranks' shards of the four linears, sequentially,
    with every host thread.  Returns (tokens/s, description, threads)."""
    from oracle import w8a8_oracle as O

    threads = torch.get_num_threads()
    sh = local_shapes(tp)
    g = torch.Generator().manual_seed(0)
    weights = {}
    for name, (n, k) in sh.items():
        weights[name] = [(torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8),
                          torch.rand(n, generator=g) * 1e-3 + 1e-5) for _ in range(1)]

    def run(m):
        x = torch.randn(m, HIDDEN, generator=g).bfloat16()
        for _r in range(tp):  # every rank's shard is the same size; rank 0's weights stand in
            wq, ws = weights["qkv"][0]
            _, _, _, qkv = O.w8a8_linear(x, wq, ws)
            attn = qkv[:, : (NQ // tp) * HEAD_DIM].contiguous()
            wq, ws = weights["o_proj"][0]
            h = O.w8a8_linear(attn, wq, ws)[3]
        h = O.all_reduce_sum([h] * tp)
        for _r in range(tp):
            wq, ws = weights["gate_up"][0]
            gu = O.w8a8_linear(h, wq, ws)[3]
            q, s, _ = O.silu_mul_quant(gu)
            wq, ws = weights["down"][0]
            out = O.dequant(O.int_gemm(q, wq), s, ws)
        return O.all_reduce_sum([out] * tp)

    m = 16
    t0 = time.perf_counter()
    run(m)
    t1 = time.perf_counter()
    per = max(t1 - t0, 1e-3)
    m = int(max(16, min(4096, m * (budget_s / 4.0) / per)))
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        run(m)
        times.append(time.perf_counter() - t0)
        if len(times) >= 10:
            break
    med = statistics.median(times)
    desc = (f"{m} tokens through all {tp} rank shard(s) of the 4 W8A8 linears + SiLU*mul quant "
            f"(oracle: torch._int_mm on CPU), median of {len(times)} runs")
    return m / med, desc, threads


def run_ours(args, rank, world, dev):
    pkg = _pkg()
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(rank, world)
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]
    comm_kind = "nccl-allreduce"
    if world > 1 and not args.nccl_baseline:
        try:
            D.enable_peer_mem_distributed(D.get_tp_info(), None, max_bytes=args.m * HIDDEN * 2, device=dev)
            comm_kind = "fused-peer-mem"
        except Exception as e:  # noqa: BLE001 - reported in the JSON
            comm_kind = f"nccl-allreduce (peer-mem unavailable: {type(e).__name__}: {e})"[:200]
    stream = torch.cuda.Stream(dev)
    flush_buf = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stack = Stack(pkg, world, rank, dev)
    pkg.ops.gemm_workspace(dev)
    peaks, peak_kind = _peaks()

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
        sweep = {}
        ops_tok, wbytes = layer_ops(world)
        for m in args.sweep:
            xm = torch.randn(m, HIDDEN, device=dev, generator=gx).bfloat16()
            tms, _, _ = time_graph(lambda: stack.forward(xm), max(20, args.steps), args.warmup, flush_buf, stream)
            tms = max_over_ranks(tms, world, dev)
            us = tms / max(20, args.steps) * 1e3
            hbm_frac = (wbytes / (us * 1e-6)) / (peaks["hbm_gbs"] * 1e9)
            sweep[str(m)] = {"tokens_per_s": round(m / (us * 1e-6), 1), "us_per_step": round(us, 2),
                             "weight_stream_frac_of_hbm": round(hbm_frac, 3)}

        # ------------------------------------------------------------ roofline: dominant kernel
        n_gu, k_gu = local_shapes(world)["gate_up"]
        qa = stack.gate_up._quantize_input(x)
        gemm_out = torch.empty(args.m, n_gu, dtype=torch.bfloat16, device=dev)
        gemm_ms = time_kernel_events(
            lambda: pkg.ops.w8a8_gemm(qa.q, stack.gate_up.weight, qa.s, stack.gate_up.weight_scale, out=gemm_out),
            max(10, args.steps // 2), flush_buf, stream)
        alg_ops = 2.0 * args.m * n_gu * k_gu
        achieved_tops = alg_ops / (gemm_ms * 1e-3) / 1e12
        peak_tops = 2.0 * peaks["bf16_tflops"]
        # library int8 yardstick on the same shape (cuBLASLt through torch._int_mm)
        try:
            wt = stack.gate_up.weight.t()
            int_mm_ms = time_kernel_events(lambda: torch._int_mm(qa.q, wt), 10, flush_buf, stream)
            int_mm_tops = alg_ops / (int_mm_ms * 1e-3) / 1e12
        except Exception:
            int_mm_tops = None
        # the reference's own GPU path for one linear: cuBLAS bf16 F.linear
        wbf = torch.randn(n_gu, k_gu, device=dev, dtype=torch.bfloat16)
        bf16_ms = time_kernel_events(lambda: torch.nn.functional.linear(x, wbf), 10, flush_buf, stream)
        del wbf
    clocks = clk.summary()

    # ---------------------------------------------------------------- e2e (public API, host buffers)
    x_host = torch.randn(args.m, HIDDEN, generator=torch.Generator().manual_seed(1)).bfloat16().pin_memory()
    y_host = torch.empty(args.m, HIDDEN, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(5, args.steps // 2)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            xd = x_host.to(dev, non_blocking=True)
            y_host.copy_(stack.forward(xd), non_blocking=True)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(e2e_steps):
            xd = x_host.to(dev, non_blocking=True)
            y_host.copy_(stack.forward(xd), non_blocking=True)
        e.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s.elapsed_time(e), world, dev)
    e2e_value = args.m * e2e_steps / (e2e_ms / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, desc, th = cpu_oracle_sample(world)
        cpu = {"value": round(v, 1), "unit": UNIT, "cores": th, "kind": "port", "sample": desc}

    traffic = _read_traffic(args.m, n_gu, k_gu)
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
        "data": "synthetic: seeded N(0,1) bf16 activations, N(0,0.02) bf16 weights quantised per channel",
        "config": {"workload": "cfg3 Qwen3-32B decoder-layer W8A8 linears, TP=N, headline M = prefill chunk",
                   "M": args.m, "hidden": HIDDEN, "heads": [NQ, NKV], "head_dim": HEAD_DIM,
                   "intermediate": INTER, "parallelism": f"tp{world}", "allreduce": comm_kind,
                   "l2": "flushed (256 MB write) before every timed step; per-step CUDA-event timing of a CUDA-graph replay"},
        "roofline": {"kernel": f"w8a8_gemm gate_up M={args.m} N={n_gu} K={k_gu}", "bound": "tensor",
                     "achieved": round(achieved_tops, 1), "peak": round(peak_tops, 1), "unit": "TOP/s (int8)",
                     "frac": round(achieved_tops / peak_tops, 4),
                     "peak_source": f"2 x {peak_kind} dense bf16 ({peaks['bf16_tflops']} TF/s burst, MEASURED_PEAKS.json): "
                                    "B200 dense int8 rate = 2 x bf16",
                     "frac_of_nominal_int8_4500": round(achieved_tops / INT8_NOMINAL_TOPS, 4),
                     "launch_ms": round(gemm_ms, 4), "traffic": traffic,
                     "algorithmic_bytes": args.m * k_gu + n_gu * k_gu + 2 * args.m * n_gu + 4 * args.m + 4 * n_gu},
        "yardsticks": {"torch_int_mm_tops_same_shape": None if int_mm_tops is None else round(int_mm_tops, 1),
                       "cublas_bf16_linear_ms_same_shape": round(bf16_ms, 4),
                       "ours_gemm_ms_same_shape": round(gemm_ms, 4)},
        "sweep": sweep,
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": args.m * HIDDEN * 2,
                "d2h_bytes_per_step": args.m * HIDDEN * 2,
                "how": "eager public layer API on the caller stream; pinned host input copied in and output copied out every step"},
        "gpu_launches": Stack.launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    return line


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    v, desc, th = cpu_oracle_sample(world, budget_s=max(5.0, min(60.0, 3.0 * args.steps)))
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(v, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": None,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 (int32 accumulate, fp32 dequant, bf16 out)",
        "data": "synthetic: seeded int8 weights and bf16 activations of the same shapes",
        "config": {"workload": "cfg3 Qwen3-32B decoder-layer W8A8 linears, TP=N", "parallelism": f"tp{world}",
                   "implementation": "CPU restatement of the reference path (oracle/w8a8_oracle.py) on host cores"},
        "cpu_baseline": {"value": round(v, 1), "unit": UNIT, "cores": th, "kind": "port", "sample": desc},
        "e2e": {"value": round(v, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--sweep", type=lambda s: [int(v) for v in s.split(",") if v], default=[1, 32, 128, 256])
    ap.add_argument("--nccl-baseline", action="store_true", help="row-parallel reduce through NCCL instead of fused")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--clocks-dir", default=tempfile.gettempdir(),
                    help="where the raw nvidia-smi samples of the timed region are written")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

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
    if args.kernel_only:
        run_kernel_only(args, dev)
        return
    if world > 1:
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=timedelta(seconds=120))
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
