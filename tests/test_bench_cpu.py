"""CPU: the parts of ``bench.py`` that need no GPU -- the cfg3 shard shapes
per TP size, the traffic figure taken from the committed ncu summary, and the
reference arm's JSON line (the CPU restatement of the reference path, which
the driver runs beside the GPU arm)."""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT


@pytest.fixture(scope="module")
def bench():
    # imported by name (the repository root is on sys.path): the CPU baseline
    # spawns ranks that must import the same module
    return importlib.import_module("bench")


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_cfg3_shard_shapes(bench, tp):
    """qkv (M, 5120, 10240/p), o (M, 8192/p, 5120), gate_up (M, 5120, 51200/p),
    down (M, 25600/p, 5120): (N, K) per rank."""
    sh = bench.local_shapes(tp)
    assert sh["qkv"] == (10240 // tp, 5120)
    assert sh["o_proj"] == (5120, 8192 // tp)
    assert sh["gate_up"] == (51200 // tp, 5120)
    assert sh["down"] == (5120, 25600 // tp)


def test_traffic_scales_with_the_shard(bench):
    full = bench._read_traffic(4096, 51200, 5120)
    assert full is not None and full > 0
    assert bench._read_traffic(4096, 12800, 5120) == round(full / 4)
    assert bench._read_traffic(128, 51200, 5120) is None


def test_reference_arm_json_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                          "--m", "64"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["unit"] == line["cpu_baseline"]["unit"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"]
    # the same workload keys as the GPU arm's config, exactly M tokens
    assert line["config"]["M"] == 64 and line["config"]["parallelism"] == "tp1"
    assert set(line["config"]) == {"workload", "M", "hidden", "heads", "head_dim", "intermediate", "layers",
                                   "parallelism"}
    assert line["cpu_baseline"]["c0_reference_bf16"]["value"] > 0


@pytest.mark.parametrize("workload,tp,shapes", [
    ("cfg2", 1, {"gate_up": (24576, 4096), "down": (4096, 12288)}),
    ("cfg4", 8, {"qkv": (1280, 8192), "o_proj": (8192, 1024), "gate_up": (7168, 8192), "down": (8192, 3584)}),
])
def test_workload_shard_shapes(bench, workload, tp, shapes):
    """BASELINE config 2 (Qwen3-8B MLP) and config 4 (Llama-3.1-70B, 4 layers
    at TP=8): the per-rank (N, K) of every linear and the step's work."""
    try:
        bench.select_workload(workload)
        assert bench.local_shapes(tp) == shapes
        ops, wbytes = bench.layer_ops(tp)
        layers = bench.WORKLOADS[workload]["layers"]
        assert ops == layers * sum(2 * n * k for n, k in shapes.values())
        assert wbytes == layers * sum(n * k + 4 * n for n, k in shapes.values())
    finally:
        bench.select_workload("cfg3")


def test_reference_arm_other_workload():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "cfg2", "--m", "32"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["config"]["hidden"] == 4096 and line["config"]["M"] == 32 and line["value"] > 0
    assert "Qwen3-8B" in line["metric"]


def test_cpu_baseline_two_gloo_ranks(bench):
    """At TP = 2 the CPU path runs as two gloo ranks whose row-parallel
    partials meet in all_reduce, at exactly M tokens."""
    cpu = bench.cpu_tp_baseline(2, 32, 2)
    assert cpu["value"] > 0 and cpu["cores"] == 2 and "TP=2" in cpu["sample"] and "M=32" in cpu["sample"]


def test_sample_rows_cover_every_tile(bench):
    for m in (1, 7, 128, 300, 4096, 8192):
        rows = bench.sample_rows(m)
        assert rows == sorted(set(rows)) and all(0 <= r < m for r in rows)
        assert {r // 128 for r in rows} == set(range((m + 127) // 128))
        assert m - 1 in rows


def _mini_bench(bench, monkeypatch):
    """Shrink the workload to a miniature layer so the oracle runs in a blink."""
    monkeypatch.setattr(bench, "HIDDEN", 64)
    monkeypatch.setattr(bench, "HEAD_DIM", 16)
    monkeypatch.setattr(bench, "NQ", 8)
    monkeypatch.setattr(bench, "NKV", 2)
    monkeypatch.setattr(bench, "INTER", 96)
    monkeypatch.setattr(bench, "PROJ", {
        "q_proj": ("self_attn", 128, 64), "k_proj": ("self_attn", 32, 64), "v_proj": ("self_attn", 32, 64),
        "o_proj": ("self_attn", 64, 128), "gate_proj": ("mlp", 96, 64), "up_proj": ("mlp", 96, 64),
        "down_proj": ("mlp", 64, 96)})


def _oracle_traces(bench, O, tp, m):
    """What collect_trace gathers, produced by the oracle itself (standing in
    for the GPU): per rank, the sampled rows of every layer."""
    dev = torch.device("cpu")
    W = {n: O.quant_weight_per_channel(bench.full_weight(n, dev)) for n in bench.PROJ}

    def sh(n, r):
        return O.shard_tensor("." + n, W[n][0], r, tp, bench.NKV), O.shard_scale("." + n, W[n][1], r, tp, bench.NKV)

    x = torch.randn(m, bench.HIDDEN, generator=torch.Generator().manual_seed(0)).bfloat16()
    qc = bench.NQ // tp * bench.HEAD_DIM
    traces = []
    for r in range(tp):
        parts = [sh(n, r) for n in ("q_proj", "k_proj", "v_proj")]
        wq, ws = torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])
        qkv = O.w8a8_linear(x, wq, ws)[3]
        xq, xs = O.quant_per_token(x)
        traces.append({"x": x, "qkv": qkv, "attn": qkv[:, :qc], "xq": xq, "xs": xs, "wq_qkv_head": wq[:4],
                       "ws_qkv": ws, "gu_again_equal": True})
    attn_full = torch.cat([t["attn"] for t in traces], dim=1)
    h = O.tp_linear("row", attn_full, W["o_proj"][0], W["o_proj"][1], tp, key=".o_proj")[0]
    parts = []
    for r, t in enumerate(traces):
        g, u = sh("gate_proj", r), sh("up_proj", r)
        _, _, acc, gu = O.w8a8_linear(h, torch.cat([g[0], u[0]]), torch.cat([g[1], u[1]]))
        q, s, _ = O.silu_mul_quant(gu)
        t.update(h=h, gu=gu, gu_i32=acc, q=q, s=s)
        parts.append(O.dequant(O.int_gemm(q, sh("down_proj", r)[0]), s, W["down_proj"][1]))
    out = O.all_reduce_sum(parts) if tp > 1 else parts[0]
    for t in traces:
        t["out"] = out.clone()
    return traces


@pytest.mark.parametrize("tp", [1, 2])
def test_oracle_parity_plumbing(bench, oracle, monkeypatch, tp):
    """oracle_parity recomputes every layer from the traced inputs: on traces
    that are right it reports bit-exact; a mistake planted in one rank's
    down output (or int32 accumulator) is reported."""
    _mini_bench(bench, monkeypatch)
    traces = _oracle_traces(bench, oracle, tp, 9)
    res = bench.oracle_parity(traces, tp, torch.device("cpu"))
    assert res["ok"] and res["bf16"] == "bit-exact" and res["int32"] == "bit-exact", res
    assert res["int8"] == "bit-exact" and res["rows"] == 9 and not res["failures"]
    traces[tp - 1]["out"] = traces[tp - 1]["out"].clone()
    traces[tp - 1]["out"][3, 5] += 1.0
    traces[0]["gu_i32"] = traces[0]["gu_i32"].clone()
    traces[0]["gu_i32"][0, 0] += 1
    res = bench.oracle_parity(traces, tp, torch.device("cpu"))
    assert not res["ok"] and res["int32"] == "mismatch" and res["bf16"] != "bit-exact"
    assert any(f.startswith(f"down+allreduce r{tp - 1}") for f in res["failures"])
