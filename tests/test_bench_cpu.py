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

from conftest import ROOT


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("w8a8_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


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
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["unit"] == line["cpu_baseline"]["unit"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"]
