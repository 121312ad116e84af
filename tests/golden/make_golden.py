"""Generate the golden fixtures in this directory from the mini-sglang reference.

Run once, in a container where the reference source tree is present::

    python tests/golden/make_golden.py --reference <path to mini-sglang>/python

It imports the reference's own Python (CPU-runnable parts only) and records
its outputs, so the oracle and the CUDA path can be checked against them on
machines where the reference is absent.  Fixtures written:

* ``shard_layout.pt``   — ``_shard_tensor`` (``M/models/weight.py:34-52``) of
  seeded q/k/v/gate/up/o/down tensors at tp = 1, 2, 4, 8, including the
  KV-head replication case (num_kv_heads < tp).
* ``layer_sizes.json``  — local input/output sizes of the five linear classes
  (``M/layers/linear.py:35-127``) for every BASELINE shape at tp = 1, 2, 4, 8,
  plus the state-dict keys each class exposes (``M/layers/base.py:19-30``).
* ``bf16_forward_exact.pt`` — the reference layers' bf16 ``forward`` on
  quantisation-exact inputs (per rank, per tp), where the W8A8 path must
  agree bit for bit.
* ``allreduce_known.pt`` — the reference's ``TorchDistributedImpl.all_reduce``
  (``M/distributed/impl.py:24-31``) run on gloo CPU ranks with the known-answer
  inputs of ``tests/kernel/test_comm.py:96-135``.
* ``w8a8_small.pt``     — oracle W8A8 vectors on small odd shapes (these pin the
  CUDA path to the oracle; the reference has no W8A8 arithmetic).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _reset_tp(r: int, n: int) -> None:
    import minisgl.distributed.info as info

    info._TP_INFO = None
    info.set_tp_info(r, n)


def make_shard_layout():
    import minisgl.models.weight as W

    g = torch.Generator().manual_seed(7)
    hd, nq, nkv, hidden, inter = 4, 8, 2, 16, 24
    tensors = {
        "model.layers.0.self_attn.q_proj.weight": torch.randn(nq * hd, hidden, generator=g),
        "model.layers.0.self_attn.k_proj.weight": torch.randn(nkv * hd, hidden, generator=g),
        "model.layers.0.self_attn.v_proj.weight": torch.randn(nkv * hd, hidden, generator=g),
        "model.layers.0.self_attn.o_proj.weight": torch.randn(hidden, nq * hd, generator=g),
        "model.layers.0.mlp.gate_proj.weight": torch.randn(inter, hidden, generator=g),
        "model.layers.0.mlp.up_proj.weight": torch.randn(inter, hidden, generator=g),
        "model.layers.0.mlp.down_proj.weight": torch.randn(hidden, inter, generator=g),
        # 1-D per-output-channel vectors follow the same positional split on dim 0
        "model.layers.0.self_attn.k_proj.bias": torch.randn(nkv * hd, generator=g),
        "model.layers.0.mlp.gate_proj.bias": torch.randn(inter, generator=g),
    }
    out = {"num_kv_heads": nkv, "inputs": tensors, "shards": {}}
    for n in (1, 2, 4, 8):
        for r in range(n):
            for k, v in tensors.items():
                out["shards"][f"{k}|{r}|{n}"] = W._shard_tensor(k, v, r, n, nkv)
    torch.save(out, os.path.join(HERE, "shard_layout.pt"))


SHAPES = {
    # name: (hidden, head_dim, nq, nkv, intermediate)
    "qwen3_0_6b": (1024, 128, 16, 8, 3072),
    "qwen3_8b": (4096, 128, 32, 8, 12288),
    "qwen3_32b": (5120, 128, 64, 8, 25600),
    "llama3_70b": (8192, 128, 64, 8, 28672),
    "qwen3_14b": (5120, 128, 40, 8, 17408),
    "kv_replicate": (256, 16, 16, 2, 512),
}


def make_layer_sizes():
    from minisgl.layers import (LinearColParallelMerged, LinearOProj, LinearQKVMerged,
                                LinearReplicated, LinearRowParallel)

    res = {}
    for name, (h, hd, nq, nkv, inter) in SHAPES.items():
        for n in (1, 2, 4, 8):
            _reset_tp(0, n)
            with torch.device("meta"):
                layers = {
                    "qkv": LinearQKVMerged(h, hd, nq, nkv, has_bias=True),
                    "o_proj": LinearOProj(nq * hd, h, has_bias=False),
                    "gate_up": LinearColParallelMerged(h, [inter, inter], has_bias=False),
                    "down": LinearRowParallel(inter, h, has_bias=False),
                    "replicated": LinearReplicated(h, 64, has_bias=True),
                }
            for lname, l in layers.items():
                res[f"{name}|{lname}|{n}"] = {
                    "full_input_size": l.full_input_size,
                    "full_output_size": l.full_output_size,
                    "local_input_size": l.local_input_size,
                    "local_output_size": l.local_output_size,
                    "state_keys": sorted(l.state_dict().keys()),
                    "weight_shape": list(l.weight.shape),
                }
    with open(os.path.join(HERE, "layer_sizes.json"), "w") as f:
        json.dump(res, f, indent=0, sort_keys=True)


def make_bf16_forward_exact():
    sys.path.insert(0, ROOT)
    from oracle.w8a8_oracle import exact_quant_inputs
    from minisgl.layers import (LinearColParallelMerged, LinearOProj, LinearQKVMerged,
                                LinearReplicated, LinearRowParallel)
    import minisgl.models.weight as W
    import torch.distributed as dist

    # world-size-1 gloo group: the row-parallel classes then return their own
    # partial (TorchDistributedImpl.all_reduce is a no-op at world size 1)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29517")
    dist.init_process_group("gloo", rank=0, world_size=1)

    hd, nq, nkv, h, inter, m = 16, 8, 2, 64, 96, 5
    cases = {}
    x, wqkv = exact_quant_inputs(m, h, (nq + 2 * nkv) * hd, seed=11)
    _, wo = exact_quant_inputs(1, nq * hd, h, seed=12)
    xo, _ = exact_quant_inputs(m, nq * hd, 1, seed=13)
    _, wgu = exact_quant_inputs(1, h, 2 * inter, seed=14)
    _, wd = exact_quant_inputs(1, inter, h, seed=15)
    xd, _ = exact_quant_inputs(m, inter, 1, seed=16)
    gb = torch.Generator().manual_seed(17)
    bias_qkv = (torch.randint(-64, 65, ((nq + 2 * nkv) * hd,), generator=gb) * 2.0 ** -6).bfloat16()
    bias_rep = (torch.randint(-64, 65, (2 * inter,), generator=gb) * 2.0 ** -6).bfloat16()

    q, k, v = wqkv.split([nq * hd, nkv * hd, nkv * hd], dim=0)
    gate, up = wgu.split([inter, inter], dim=0)
    bq, bk, bv = bias_qkv.split([nq * hd, nkv * hd, nkv * hd], dim=0)
    pre = "model.layers.0."
    for n in (1, 2, 4, 8):
        for r in range(n):
            _reset_tp(r, n)
            sh = lambda key, t: W._shard_tensor(pre + key, t, r, n, nkv)  # noqa: E731
            lq = LinearQKVMerged(h, hd, nq, nkv, has_bias=True)
            # BaseOP.load_state_dict asserts dtype equality and the classes
            # allocate fp32 placeholders, so the bf16 shards are assigned directly.
            lq.weight = torch.cat([sh("self_attn.q_proj.weight", q), sh("self_attn.k_proj.weight", k),
                                   sh("self_attn.v_proj.weight", v)], 0)
            lq.bias = torch.cat([sh("self_attn.q_proj.bias", bq), sh("self_attn.k_proj.bias", bk),
                                 sh("self_attn.v_proj.bias", bv)], 0)
            lo = LinearOProj(nq * hd, h, has_bias=False)
            lo.weight = sh("self_attn.o_proj.weight", wo)
            lgu = LinearColParallelMerged(h, [inter, inter], has_bias=False)
            lgu.weight = torch.cat([sh("mlp.gate_proj.weight", gate), sh("mlp.up_proj.weight", up)], 0)
            ld = LinearRowParallel(inter, h, has_bias=False)
            ld.weight = sh("mlp.down_proj.weight", wd)
            xo_r = xo.chunk(n, dim=1)[r].contiguous()
            xd_r = xd.chunk(n, dim=1)[r].contiguous()
            cases[f"qkv|{r}|{n}"] = dict(x=x, weight=lq.weight, bias=lq.bias, y=lq.forward(x))
            cases[f"o_proj|{r}|{n}"] = dict(x=xo_r, weight=lo.weight, bias=None, y=lo.forward(xo_r))
            cases[f"gate_up|{r}|{n}"] = dict(x=x, weight=lgu.weight, bias=None, y=lgu.forward(x))
            cases[f"down|{r}|{n}"] = dict(x=xd_r, weight=ld.weight, bias=None, y=ld.forward(xd_r))
            if n == 1:
                lr = LinearReplicated(h, 2 * inter, has_bias=True)
                lr.weight, lr.bias = wgu, bias_rep
                cases["replicated|0|1"] = dict(x=x, weight=wgu, bias=bias_rep, y=lr.forward(x))
    dist.destroy_process_group()
    torch.save({"full": dict(x=x, wqkv=wqkv, bias_qkv=bias_qkv, wo=wo, xo=xo, wgu=wgu, wd=wd,
                             xd=xd, bias_rep=bias_rep, hd=hd, nq=nq, nkv=nkv, h=h, inter=inter),
                "cases": cases}, os.path.join(HERE, "bf16_forward_exact.pt"))


def _allreduce_rank(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist
    from minisgl.distributed import DistributedCommunicator

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = DistributedCommunicator()
    n = 4096
    res = {}
    x = torch.ones(n, dtype=torch.bfloat16)
    for _ in range(4):
        x = comm.all_reduce(x)
    res["ones_pow4"] = x.clone()
    x = torch.full((n,), rank, dtype=torch.bfloat16)
    res["rank_sum"] = comm.all_reduce(x).clone()
    x = torch.cat([torch.zeros(n // 2, dtype=torch.bfloat16), torch.ones(n // 2, dtype=torch.bfloat16)])
    res["half_ones"] = comm.all_reduce(x).clone()
    q.put((rank, res))
    dist.destroy_process_group()


def make_allreduce_known():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = {}
    for i, world in enumerate((2, 4)):
        q = ctx.Queue()
        ps = [ctx.Process(target=_allreduce_rank, args=(r, world, 29600 + i, q)) for r in range(world)]
        for p in ps:
            p.start()
        got = dict(q.get(timeout=120) for _ in range(world))
        for p in ps:
            p.join(timeout=60)
        out[world] = got
    torch.save(out, os.path.join(HERE, "allreduce_known.pt"))


def make_w8a8_small():
    sys.path.insert(0, ROOT)
    from oracle import w8a8_oracle as O

    out = {}
    for (m, k, n, seed, bias) in [(1, 32, 16, 0, False), (3, 64, 48, 1, True), (17, 144, 80, 2, False),
                                  (64, 256, 272, 3, True), (130, 160, 112, 4, False)]:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(m, k, generator=g).bfloat16()
        w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
        b = (torch.randn(n, generator=g) * 0.1).bfloat16() if bias else None
        wq, ws = O.quant_weight_per_channel(w)
        xq, xs, acc, y = O.w8a8_linear(x, wq, ws, b)
        out[f"{m}x{k}x{n}"] = dict(x=x, wq=wq, ws=ws, bias=b, xq=xq, xs=xs, acc=acc, y=y)
    g = torch.Generator().manual_seed(5)
    gu = torch.randn(7, 2 * 96, generator=g).bfloat16()
    q, s, y = O.silu_mul_quant(gu)
    out["silu_mul_quant"] = dict(gate_up=gu, q=q, s=s, y=y)
    torch.save(out, os.path.join(HERE, "w8a8_small.pt"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to mini-sglang's python/ directory")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    make_shard_layout()
    make_layer_sizes()
    make_bf16_forward_exact()
    make_allreduce_known()
    make_w8a8_small()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
