"""GPU: kernel 2 (tcgen05 W8A8 GEMM) vs the CPU oracle.

The int32 accumulator must be bit-exact.  The bf16 output follows the same
separately-rounded fp32 dequant as the oracle and is asserted bit-exact too;
the north-star tolerance (1e-2 rel / 1e-2 abs) is asserted on top as the
contract bound.
"""
from __future__ import annotations

import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

RTOL = 1e-2
ATOL = 1e-2


def _operands(m, n, k, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    aq = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    wq = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sa = torch.rand(m, generator=g) * 0.02 + 1e-4
    sw = torch.rand(n, generator=g) * 0.002 + 1e-5
    b = (torch.randn(n, generator=g) * 0.5).bfloat16() if bias else None
    return aq, wq, sa, sw, b


def _check(pkg, oracle, dev, m, n, k, variant=0, ctas=0, bias=False, seed=0):
    aq, wq, sa, sw, b = _operands(m, n, k, seed, bias)
    acc_ref = oracle.int_gemm(aq, wq)
    y_ref = oracle.dequant(acc_ref, sa, sw, b)
    acc = torch.empty(m, n, dtype=torch.int32, device=dev)
    y = pkg.ops.w8a8_gemm(aq.to(dev), wq.to(dev), sa.to(dev), sw.to(dev), None if b is None else b.to(dev),
                          out_i32=acc, variant=variant, ctas=ctas)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    assert torch.equal(acc.cpu(), acc_ref), f"int32 mismatch m={m} n={n} k={k} v={variant} ctas={ctas}"
    yc = y.cpu()
    torch.testing.assert_close(yc.float(), y_ref.float(), rtol=RTOL, atol=ATOL)
    assert torch.equal(yc, y_ref), f"bf16 mismatch m={m} n={n} k={k} v={variant} ctas={ctas}"


# (m, n, k) spanning every variant's edge cases: partial tiles, K not a
# multiple of the 128-byte stage, tiny shapes.
CASES = [
    (1, 16, 16), (3, 48, 64), (17, 80, 144), (64, 272, 256), (128, 128, 128),
    (130, 112, 160), (200, 512, 384), (257, 784, 1040), (64, 6144, 1024),
]


@pytest.mark.parametrize("variant", [1, 2, 3, 4, 5, 6, 7])
@pytest.mark.parametrize("m,n,k", CASES)
def test_gemm_variants_bit_exact(pkg, oracle, cuda_dev, variant, m, n, k):
    _check(pkg, oracle, cuda_dev, m, n, k, variant=variant, seed=m + n + k + variant)


@pytest.mark.parametrize("variant", [1, 2, 3, 5, 6])
@pytest.mark.parametrize("ctas", [1, 2, 3, 7, 64])
def test_gemm_stream_k_bit_exact(pkg, oracle, cuda_dev, variant, ctas):
    """Few CTAs over many tiles: ranges cut tiles at arbitrary k blocks, and a
    tile can be shared by several CTAs (workspace fix-up path)."""
    _check(pkg, oracle, cuda_dev, 40, 400, 1024, variant=variant, ctas=ctas, seed=ctas * 10 + variant)
    _check(pkg, oracle, cuda_dev, 130, 272, 1664, variant=variant, ctas=ctas, seed=ctas * 10 + variant + 1)


@pytest.mark.parametrize("m,n,k", [(1, 24576, 4096), (16, 4096, 12288), (64, 6144, 1024), (256, 5120, 8192),
                                   (2048, 2048, 4096), (33, 1280, 8192),
                                   # stream-K remainder smaller than the grid (160 tiles, 148 CTAs, 4 k blocks)
                                   (1024, 5120, 512), (1100, 5120, 256)])
def test_gemm_auto_plan(pkg, oracle, cuda_dev, m, n, k):
    _check(pkg, oracle, cuda_dev, m, n, k, bias=(m % 2 == 0), seed=m * 3 + n)


@pytest.mark.parametrize("ctas", [2, 6, 148])
@pytest.mark.parametrize("m,n,k", [(384, 768, 640), (1000, 1040, 256), (256, 256, 128)])
def test_gemm_pair_variant_bit_exact(pkg, oracle, cuda_dev, m, n, k, ctas):
    """2-SM (CTA pair) variant: odd 128-row tile counts (a phantom half), N not
    a multiple of 256, K tails, few or many pairs."""
    _check(pkg, oracle, cuda_dev, m, n, k, variant=7, ctas=ctas, bias=(m % 2 == 0), seed=m + ctas)


@pytest.mark.parametrize("m,n,k,ctas", [
    (1100, 1024, 2128, 16),   # 20 blocks on 8 pairs: 4 left, split 2 (17 k blocks: 8 + 9), phantom half
    (500, 1200, 4224, 18),    # 10 blocks on 9 pairs: 1 left, split 4 (33 k blocks), N tail
    (1280, 1024, 3200, 18),   # 20 blocks on 9 pairs: 2 left, split 3 (25 k blocks; 4 would leave 6 each)
    (1280, 1024, 2176, 12),   # 20 blocks on 6 pairs: 2 left, split 2 (3 would leave 5 k blocks each)
])
def test_gemm_pair_last_wave_split(pkg, oracle, cuda_dev, m, n, k, ctas):
    """Pair variant with its last, partial wave split along K over the idle
    pairs: share j > 0 parks its int32 partial sums in the workspace, the pair
    holding share 0 adds them.  Bit-exact, and the counters return to zero."""
    p = pkg.ops.gemm_plan(m, n, k, variant=7, ctas=ctas,
                          num_sms=torch.cuda.get_device_properties(0).multi_processor_count)
    assert p["workspace_bytes"] > 0   # the split is planned
    for rep in range(2):
        _check(pkg, oracle, cuda_dev, m, n, k, variant=7, ctas=ctas, bias=(rep == 1), seed=m + k + rep)
    ws = pkg.ops.gemm_workspace(cuda_dev)
    assert int(ws[: 65536 * 4].count_nonzero()) == 0


def test_stream_k_counters_return_to_zero(pkg, oracle, cuda_dev):
    """Back-to-back stream-K calls of different shapes sharing the workspace:
    every call leaves the tile counters at the workspace head zeroed, and no
    call's partial tiles land on another call's counters."""
    for rep, (m, n, k) in enumerate([(5, 4096, 12288), (300, 8192, 1024), (7, 2048, 3072), (5, 4096, 12288)]):
        _check(pkg, oracle, cuda_dev, m, n, k, seed=rep)
    p = pkg.ops.gemm_plan(5, 4096, 12288, num_sms=torch.cuda.get_device_properties(0).multi_processor_count)
    assert p["workspace_bytes"] > 0
    ws = pkg.ops.gemm_workspace(cuda_dev)
    assert int(ws[: 65536 * 4].count_nonzero()) == 0   # the whole fixed counter region


def test_gemm_golden_small(pkg, oracle, cuda_dev):
    d = golden("w8a8_small.pt")
    for key, c in d.items():
        if key == "silu_mul_quant":
            continue
        dev = cuda_dev
        xq, xs = pkg.ops.quant_per_token(c["x"].to(dev))
        assert torch.equal(xq.cpu(), c["xq"]) and torch.equal(xs.cpu(), c["xs"]), key
        n = c["wq"].shape[0]
        if n % 16 or c["x"].shape[1] % 16:
            continue
        acc = torch.empty(c["acc"].shape, dtype=torch.int32, device=dev)
        y = pkg.ops.w8a8_gemm(xq, c["wq"].to(dev), xs, c["ws"].to(dev),
                              None if c["bias"] is None else c["bias"].to(dev), out_i32=acc)
        assert torch.equal(acc.cpu(), c["acc"]), key
        assert torch.equal(y.cpu(), c["y"]), key


def test_gemm_matches_reference_bf16_forward_on_exact_inputs(pkg, oracle, cuda_dev):
    """The full GPU path (quant kernel + GEMM) reproduces the reference layers'
    bf16 F.linear outputs bit for bit on quantisation-exact inputs."""
    d = golden("bf16_forward_exact.pt")
    for key, c in d["cases"].items():
        wq, ws = oracle.quant_weight_per_channel(c["weight"])
        if wq.shape[0] % 16 or wq.shape[1] % 16:
            continue
        xq, xs = pkg.ops.quant_per_token(c["x"].to(cuda_dev))
        y = pkg.ops.w8a8_gemm(xq, wq.to(cuda_dev), xs, ws.to(cuda_dev),
                              None if c["bias"] is None else c["bias"].to(cuda_dev))
        assert torch.equal(y.cpu(), c["y"]), key


def test_gemm_empty_batch(pkg, cuda_dev):
    aq = torch.empty(0, 64, dtype=torch.int8, device=cuda_dev)
    wq = torch.zeros(32, 64, dtype=torch.int8, device=cuda_dev)
    y = pkg.ops.w8a8_gemm(aq, wq, torch.empty(0, device=cuda_dev), torch.ones(32, device=cuda_dev))
    assert y.shape == (0, 32)


def test_gemm_extreme_values(pkg, oracle, cuda_dev):
    """All-(-127) operands: the largest int32 magnitudes the K range produces."""
    m, n, k = 24, 64, 16384
    aq = torch.full((m, k), -127, dtype=torch.int8)
    wq = torch.full((n, k), -127, dtype=torch.int8)
    wq[1::2] = 127
    sa = torch.full((m,), 1e-3)
    sw = torch.full((n,), 1e-3)
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda_dev)
    y = pkg.ops.w8a8_gemm(aq.to(cuda_dev), wq.to(cuda_dev), sa.to(cuda_dev), sw.to(cuda_dev), out_i32=acc)
    ref = oracle.int_gemm(aq, wq)
    assert torch.equal(acc.cpu(), ref)
    assert torch.equal(y.cpu(), oracle.dequant(ref, sa, sw))


def test_gemm_rejects_bad_shapes_without_launch(pkg, cuda_dev):
    aq = torch.zeros(4, 24, dtype=torch.int8, device=cuda_dev)
    wq = torch.zeros(32, 24, dtype=torch.int8, device=cuda_dev)
    with pytest.raises(pkg.W8A8Error, match="multiple of 16"):
        pkg.ops.w8a8_gemm(aq, wq, torch.ones(4, device=cuda_dev), torch.ones(32, device=cuda_dev))


def test_gemm_workspace_reset_clears_stale_counters(pkg, oracle, cuda_dev):
    """A call whose bounded wait gave up can leave stream-K tile counters
    non-zero.  reset_gemm_workspace (run by device_error when it clears a
    non-zero error word) zeroes them, after which a cut-tile GEMM on the same
    workspace matches the oracle and leaves the counters at zero again."""
    ws = pkg.ops.gemm_workspace(cuda_dev)
    assert pkg.ops.gemm_plan(40, 400, 1024, variant=2, ctas=7)["workspace_bytes"] > 0  # tiles are cut
    ws[: 64 * 4].fill_(1)  # stale counters, written from the host side
    pkg.ops.reset_gemm_workspace(cuda_dev)
    _check(pkg, oracle, cuda_dev, 40, 400, 1024, variant=2, ctas=7, seed=11)
    assert int(ws[: pkg.ops._COUNTER_BYTES].count_nonzero()) == 0


def _tile_rows(m):
    """Two rows of every 128-row tile (one pseudo-random, the tile's last)."""
    rows = set()
    for t in range((m + 127) // 128):
        lo, hi = t * 128, min(m, t * 128 + 128)
        rows.update((lo + (t * 53 + 17) % (hi - lo), hi - 1))
    return sorted(rows)


# The benchmarked shapes: every cfg3 shard (qkv, o_proj, gate_up, down) at the
# M = 4096 prefill chunk for TP 1/2/4/8, and two M = 8192 prefill shapes
# (cfg2 gate_up and down).
HEADLINE_SHAPES = sorted({(4096, n, k) for p in (1, 2, 4, 8)
                          for n, k in ((10240 // p, 5120), (5120, 8192 // p), (51200 // p, 5120), (5120, 25600 // p))}
                         | {(8192, 24576, 4096), (8192, 4096, 12288)})


@pytest.mark.parametrize("m,n,k", HEADLINE_SHAPES)
def test_gemm_headline_shapes(pkg, oracle, cuda_dev, m, n, k):
    """Auto-planned GEMM at the exact shapes the bench times: the sampled rows
    (every output tile) bit-exact in int32 and bf16 against the oracle, and
    every row through the column-checksum identity
    sum_m acc[m, n] == (sum_m a[m, :]) . w[n, :] in int64."""
    g = torch.Generator(device=cuda_dev).manual_seed(m * 7 + n * 3 + k)
    a = torch.randint(-127, 128, (m, k), device=cuda_dev, generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), device=cuda_dev, generator=g, dtype=torch.int8)
    sa = torch.rand(m, device=cuda_dev, generator=g) * 0.02 + 1e-4
    sw = torch.rand(n, device=cuda_dev, generator=g) * 0.002 + 1e-5
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda_dev)
    y = pkg.ops.w8a8_gemm(a, w, sa, sw, out_i32=acc)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    plan = pkg.ops.gemm_plan(m, n, k)
    rows = torch.tensor(_tile_rows(m), device=cuda_dev)
    a_r, w_c = a.index_select(0, rows).cpu(), w.cpu()
    acc_ref = oracle.int_gemm(a_r, w_c)
    y_ref = oracle.dequant(acc_ref, sa.index_select(0, rows).cpu(), sw.cpu())
    assert torch.equal(acc.index_select(0, rows).cpu(), acc_ref), f"int32 rows, plan {plan}"
    assert torch.equal(y.index_select(0, rows).cpu(), y_ref), f"bf16 rows, plan {plan}"
    col = acc.sum(dim=0, dtype=torch.int64).cpu()
    want = (a.sum(dim=0, dtype=torch.int64).cpu().numpy() @ w_c.numpy().astype("int64").T)
    assert torch.equal(col, torch.from_numpy(want)), f"column checksum, plan {plan}"
