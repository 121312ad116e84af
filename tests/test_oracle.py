"""CPU: the oracle pinned against the reference's own outputs (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py`` importing the
mini-sglang reference: ``_shard_tensor`` (M/models/weight.py:34-52), the bf16
layers' ``forward`` (M/layers/linear.py:13-127) on quantisation-exact inputs,
and ``TorchDistributedImpl.all_reduce`` (M/distributed/impl.py:24-31) on the
known answers of tests/kernel/test_comm.py:96-135.
"""
from __future__ import annotations

import pytest
import torch

from conftest import golden


def test_shard_layout_matches_reference(oracle):
    g = golden("shard_layout.pt")
    nkv = g["num_kv_heads"]
    assert len(g["shards"]) > 0
    for key, ref in g["shards"].items():
        name, r, n = key.split("|")
        got = oracle.shard_tensor(name, g["inputs"][name], int(r), int(n), nkv)
        assert torch.equal(got, ref), key


def test_int8_weight_shards_follow_bf16_layout(oracle):
    """Quantise-then-shard equals shard-then-take-the-rows for dim-0 splits,
    and dim-1 shards keep the full-row scale (replicated)."""
    g = golden("shard_layout.pt")
    nkv = g["num_kv_heads"]
    for name, w in g["inputs"].items():
        if w.dim() != 2:
            continue
        q, s = oracle.quant_weight_per_channel(w.bfloat16())
        for n in (2, 4, 8):
            for r in range(n):
                qs = oracle.shard_tensor(name, q, r, n, nkv)
                ss = oracle.shard_scale(name, s, r, n, nkv)
                assert qs.shape[0] == ss.shape[0]
                if ".o_proj" in name or ".down_proj" in name:
                    assert torch.equal(ss, s)
                else:
                    ws = oracle.shard_tensor(name, w.bfloat16(), r, n, nkv)
                    q2, s2 = oracle.quant_weight_per_channel(ws)
                    assert torch.equal(qs, q2) and torch.equal(ss, s2)


def test_layer_local_sizes_match_reference(oracle):
    import json
    import os

    from conftest import GOLDEN

    with open(os.path.join(GOLDEN, "layer_sizes.json")) as f:
        ref = json.load(f)
    shapes = {"qwen3_0_6b": (1024, 128, 16, 8, 3072), "qwen3_8b": (4096, 128, 32, 8, 12288),
              "qwen3_32b": (5120, 128, 64, 8, 25600), "llama3_70b": (8192, 128, 64, 8, 28672),
              "qwen3_14b": (5120, 128, 40, 8, 17408), "kv_replicate": (256, 16, 16, 2, 512)}
    for key, want in ref.items():
        name, lname, n = key.split("|")
        h, hd, nq, nkv, inter = shapes[name]
        n = int(n)
        if lname == "qkv":
            got = oracle.local_sizes("qkv", n, hidden_size=h, head_dim=hd, num_qo_heads=nq, num_kv_heads=nkv)
        elif lname == "o_proj":
            got = oracle.local_sizes("o_proj", n, input_size=nq * hd, output_size=h)
        elif lname == "gate_up":
            got = oracle.local_sizes("col_merged", n, input_size=h, output_sizes=[inter, inter])
        elif lname == "down":
            got = oracle.local_sizes("row", n, input_size=inter, output_size=h)
        else:
            got = oracle.local_sizes("replicated", n, input_size=h, output_size=64)
        assert got == (want["full_input_size"], want["full_output_size"], want["local_input_size"],
                       want["local_output_size"]), key


def test_w8a8_equals_reference_bf16_forward_on_exact_inputs(oracle):
    """On quantisation-exact inputs W8A8 is lossless, so the oracle must equal
    the reference layers' bf16 F.linear output bit for bit — every class, every
    rank, tp = 1, 2, 4, 8."""
    d = golden("bf16_forward_exact.pt")
    assert len(d["cases"]) == 61
    for key, c in d["cases"].items():
        wq, ws = oracle.quant_weight_per_channel(c["weight"])
        _, _, acc, y = oracle.w8a8_linear(c["x"], wq, ws, c["bias"])
        assert torch.equal(y, c["y"]), key
        assert torch.equal(acc.to(torch.int64), oracle.int_gemm_int64(*oracle.quant_per_token(c["x"])[:1], wq))


def test_row_parallel_sum_matches_reference_partials(oracle):
    """TP row-parallel: the oracle's reduced output equals the fp32 sum of the
    reference layers' per-rank bf16 partials."""
    d = golden("bf16_forward_exact.pt")
    full = d["full"]
    for lname, xkey, wkey in (("o_proj", "xo", "wo"), ("down", "xd", "wd")):
        for n in (2, 4, 8):
            parts = [d["cases"][f"{lname}|{r}|{n}"]["y"] for r in range(n)]
            want = oracle.all_reduce_sum(parts)
            wq, ws = oracle.quant_weight_per_channel(full[wkey])
            key = ".o_proj" if lname == "o_proj" else ".down_proj"
            got = oracle.tp_linear("row", full[xkey], wq, ws, n, key=key)
            for y in got:
                assert torch.equal(y, want), (lname, n)


def test_all_reduce_known_answers(oracle):
    """tests/kernel/test_comm.py:96-135 known answers, from the reference's own
    all_reduce on gloo ranks, reproduced by the oracle's rank-order fp32 sum."""
    d = golden("allreduce_known.pt")
    for world, ranks in d.items():
        n = ranks[0]["ones_pow4"].numel()
        x = [torch.ones(n, dtype=torch.bfloat16) for _ in range(world)]
        for _ in range(4):
            y = oracle.all_reduce_sum(x)
            x = [y.clone() for _ in range(world)]
        rank_sum = oracle.all_reduce_sum([torch.full((n,), r, dtype=torch.bfloat16) for r in range(world)])
        half = torch.cat([torch.zeros(n // 2), torch.ones(n // 2)]).bfloat16()
        half_sum = oracle.all_reduce_sum([half] * world)
        for r in range(world):
            assert torch.equal(x[r], ranks[r]["ones_pow4"])
            assert torch.equal(rank_sum, ranks[r]["rank_sum"])
            assert torch.equal(half_sum, ranks[r]["half_ones"])
        assert float(x[0][0]) == world ** 4
        assert float(rank_sum[0]) == world * (world - 1) // 2


def test_w8a8_small_goldens_reproduce(oracle):
    d = golden("w8a8_small.pt")
    for key, c in d.items():
        if key == "silu_mul_quant":
            q, s, y = oracle.silu_mul_quant(c["gate_up"])
            assert torch.equal(q, c["q"]) and torch.equal(s, c["s"]) and torch.equal(y, c["y"])
            continue
        xq, xs, acc, y = oracle.w8a8_linear(c["x"], c["wq"], c["ws"], c["bias"])
        assert torch.equal(xq, c["xq"]) and torch.equal(xs, c["xs"])
        assert torch.equal(acc, c["acc"]) and torch.equal(y, c["y"])
        assert torch.equal(acc.to(torch.int64), oracle.int_gemm_int64(xq, c["wq"]))


def test_quant_convention_edges(oracle):
    x = torch.zeros(3, 16, dtype=torch.bfloat16)
    x[1, 3] = 2.0
    x[1, 4] = -1.0
    x[2] = torch.linspace(-5, 5, 16).bfloat16()
    q, s = oracle.quant_per_token(x)
    assert s[0] == 0 and torch.all(q[0] == 0)          # all-zero row -> scale 0, q 0
    assert q[1, 3] == 127 and q[1, 4] in (-63, -64)     # -1 / (2/127) ~= -63.5
    assert q.abs().max() <= 127
    assert torch.equal(s, x.float().abs().amax(1) / 127.0)
    # round-half-even on exact halves
    y = torch.tensor([[127.0, 0.5, 1.5, 2.5, -0.5, -1.5, 3.5, 0.0]], dtype=torch.bfloat16)
    qy, sy = oracle.quant_per_token(y)
    assert float(sy[0]) == 1.0
    assert qy[0].tolist() == [127, 0, 2, 2, 0, -2, 4, 0]


@pytest.mark.parametrize("m,k,n", [(1, 16, 16), (7, 48, 32), (33, 128, 80)])
def test_int_gemm_exact(oracle, m, k, n):
    g = torch.Generator().manual_seed(m * 131 + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    assert torch.equal(oracle.int_gemm(a, b).to(torch.int64), oracle.int_gemm_int64(a, b))


def test_rmsnorm_restatement_matches_torch_rms_norm(oracle):
    """The oracle's RMSNorm (fp32, correctly rounded 1/sqrt) against torch's
    own fp32 rms_norm, before the common bf16 rounding: same to fp32 noise."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn(16, 512, generator=g).bfloat16()
    r = torch.randn(16, 512, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(512, generator=g)).bfloat16()
    y, res = oracle.rmsnorm(x, w, 1e-6, r)
    v = x.float() + r.float()
    ref = torch.nn.functional.rms_norm(v, (512,), w.float(), 1e-6)
    assert torch.equal(res, v.bfloat16())
    torch.testing.assert_close(y.float(), ref, atol=0, rtol=2 ** -7)
    q, s, y2, res2 = oracle.rmsnorm_quant(x, w, 1e-6)
    assert res2 is x and torch.equal(y2, oracle.rmsnorm(x, w, 1e-6)[0])
    assert torch.equal((q, s)[0], oracle.quant_per_token(y2)[0])
