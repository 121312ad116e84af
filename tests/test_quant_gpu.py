"""GPU: kernel 1 (per-token quantiser, fused SiLU*mul+quant) vs the CPU oracle.

int8 values and fp32 scales must be bit-exact.  The fused kernel's bf16 SiLU
product may differ from the CPU's in the last bit (its exp is 2^(x log2 e) on
the ex2 unit, ~1e-6 relative at worst); it is checked within 1 bf16 ulp
(rel 2**-7) on every element and bit-exact on all but 0.1 % of them, and its
quantisation is checked bit-exact against the oracle applied to the kernel's
own bf16 product.
"""
from __future__ import annotations

import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

SHAPES = [(1, 8), (1, 4096), (3, 24), (17, 1024), (64, 1024), (130, 5120), (257, 12288), (5, 28672), (33, 25600)]


def _x(m, k, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(m, k, generator=g) * scale).bfloat16()


@pytest.mark.parametrize("m,k", SHAPES)
def test_quant_per_token_bit_exact(pkg, oracle, cuda_dev, m, k):
    x = _x(m, k, seed=m * 7 + k)
    q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
    qr, sr = oracle.quant_per_token(x)
    assert torch.equal(s.cpu(), sr)
    assert torch.equal(q.cpu(), qr)


def test_quant_edge_rows(pkg, oracle, cuda_dev):
    x = _x(6, 256, seed=3, scale=30.0)
    x[0] = 0                                   # all-zero row: scale 0, q 0
    x[1, :] = 1e-30                            # tiny values
    x[2, 5] = 3.0e38                           # near bf16 max
    x[3] = torch.linspace(-127, 127, 256).round().bfloat16()   # exact halves / integers
    x[4, :128] = 0.5
    x[4, 128] = 127                            # scale exactly 1 -> 0.5 rounds to even 0
    q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
    qr, sr = oracle.quant_per_token(x)
    assert torch.equal(s.cpu(), sr) and torch.equal(q.cpu(), qr)
    assert float(s[0]) == 0.0 and int(q[0].abs().max()) == 0
    assert int(q[4, 0]) == 0


def test_quant_half_integer_ties(pkg, oracle, cuda_dev):
    """x / s at or next to a half-integer: the kernel's reciprocal fast path
    must fall back to the exact quotient there and round half to even."""
    rows = []
    ties = torch.arange(0, 127).float() + 0.5                        # s == 1: exact ties
    rows.append(torch.cat([torch.tensor([127.0]), ties, -ties, torch.zeros(1)]).bfloat16())  # 256 wide
    g = torch.Generator().manual_seed(1)
    for _ in range(63):
        amax = float(torch.rand(1, generator=g)) * 10 + 0.01
        s = torch.tensor(amax, dtype=torch.float32) / 127.0
        k = torch.randint(-127, 127, (255,), generator=g).float() + 0.5
        near = (k * s).bfloat16()                                       # bf16 values close to ties
        rows.append(torch.cat([torch.tensor([amax]).bfloat16(), near]))
    x = torch.stack(rows)
    q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
    qr, sr = oracle.quant_per_token(x)
    assert torch.equal(s.cpu(), sr) and torch.equal(q.cpu(), qr)
    assert q[0, 1:5].tolist() == [0, 2, 2, 4]


def test_quant_strided_rows(pkg, oracle, cuda_dev):
    """A row-strided view (e.g. a slice of a wider buffer) quantises like its copy."""
    big = _x(9, 512, seed=11).to(cuda_dev)
    view = big[:, 128:384]
    q, s = pkg.ops.quant_per_token(view)
    qr, sr = oracle.quant_per_token(view.cpu())
    assert torch.equal(q.cpu(), qr) and torch.equal(s.cpu(), sr)


def test_quant_empty_batch(pkg, cuda_dev):
    q, s = pkg.ops.quant_per_token(torch.empty(0, 64, dtype=torch.bfloat16, device=cuda_dev))
    assert q.shape == (0, 64) and s.shape == (0,)


@pytest.mark.parametrize("m,i", [(1, 8), (7, 96), (64, 3072), (5, 12288), (33, 6400), (2, 14336)])
def test_silu_mul_quant(pkg, oracle, cuda_dev, m, i):
    gu = _x(m, 2 * i, seed=m + i, scale=2.0)
    qa, y = pkg.ops.silu_and_mul_quant(gu.to(cuda_dev), with_bf16=True)
    y_ref = oracle.silu_and_mul(gu)
    yc = y.cpu()
    # bf16 product within one bf16 ulp of the CPU reference
    diff = (yc.float() - y_ref.float()).abs()
    assert torch.all(diff <= y_ref.float().abs() * 2.0 ** -7 + 1e-30), float(diff.max())
    mismatch = (yc != y_ref).float().mean().item()
    assert mismatch < 1e-3, mismatch
    # quantisation of the kernel's own bf16 product is bit-exact
    q_ref, s_ref = oracle.quant_per_token(yc)
    assert torch.equal(qa.s.cpu(), s_ref) and torch.equal(qa.q.cpu(), q_ref)


def test_silu_mul_quant_golden(pkg, oracle, cuda_dev):
    c = golden("w8a8_small.pt")["silu_mul_quant"]
    qa, y = pkg.ops.silu_and_mul_quant(c["gate_up"].to(cuda_dev), with_bf16=True)
    q_ref, s_ref = oracle.quant_per_token(y.cpu())
    assert torch.equal(qa.q.cpu(), q_ref) and torch.equal(qa.s.cpu(), s_ref)
    assert (y.cpu().float() - c["y"].float()).abs().max() <= c["y"].float().abs().max() * 2.0 ** -7


def test_silu_and_mul_compat_signature(pkg, oracle, cuda_dev):
    gu = _x(4, 64, seed=9).to(cuda_dev)
    out = torch.empty(4, 32, dtype=torch.bfloat16, device=cuda_dev)
    y = pkg.silu_and_mul(gu, out=out)
    assert y.data_ptr() == out.data_ptr()
    torch.testing.assert_close(y.cpu(), oracle.silu_and_mul(gu.cpu()), rtol=2 ** -7, atol=0)


def test_silu_mul_extreme_gate(pkg, oracle, cuda_dev):
    """Gate values where 1 + exp(-g) lies in (2^126, 2^128) (about [-88.7,
    -87.3]; the fast divide would return 0 for a normal ~1e-36 result) and
    beyond (exp overflows: the quotient is -0): the bf16 product follows the
    CPU reference there too."""
    m, i = 3, 256
    g = torch.linspace(-89.5, -86.5, m * i).reshape(m, i)
    u = torch.full((m, i), 3.0)
    u[1] = -1.5
    gu = torch.cat([g, u], dim=1).bfloat16()
    qa, y = pkg.ops.silu_and_mul_quant(gu.to(cuda_dev), with_bf16=True)
    y_ref = oracle.silu_and_mul(gu)
    yc = y.cpu()
    diff = (yc.float() - y_ref.float()).abs()
    assert torch.all(diff <= y_ref.float().abs() * 2.0 ** -7), float(diff.max())
    assert torch.equal(yc == 0, y_ref == 0)
    q_ref, s_ref = oracle.quant_per_token(yc)
    assert torch.equal(qa.s.cpu(), s_ref) and torch.equal(qa.q.cpu(), q_ref)
    # the bf16-only form computes the same product
    torch.testing.assert_close(pkg.silu_and_mul(gu.to(cuda_dev)).cpu(), yc, rtol=0, atol=0)


@pytest.mark.parametrize("m,i", [(1, 8), (7, 96), (300, 3072), (4096, 3200)])
def test_silu_and_mul_bf16_only(pkg, oracle, cuda_dev, m, i):
    """The bf16-only silu_and_mul (no quantisation) equals the fused kernel's
    bf16 product bit for bit and is within one bf16 ulp of the CPU reference;
    it also accepts a strided gate_up view."""
    gu = _x(m, 2 * i + 16, seed=m * 3 + i, scale=2.0)[:, : 2 * i]
    gd = gu.to(cuda_dev)
    y = pkg.silu_and_mul(gd)
    _, y_fused = pkg.ops.silu_and_mul_quant(gd, with_bf16=True)
    assert torch.equal(y.cpu(), y_fused.cpu())
    y_ref = oracle.silu_and_mul(gu.contiguous())
    diff = (y.cpu().float() - y_ref.float()).abs()
    assert torch.all(diff <= y_ref.float().abs() * 2.0 ** -7 + 1e-30), float(diff.max())


# Few rows (decode): each row is split over a cluster of 2..8 CTAs whose
# absmax meets through distributed shared memory; 1..4 vectors per thread.
CLUSTER_SHAPES = [(1, 4096), (1, 5120), (1, 32768), (16, 5120), (32, 8192), (37, 25600), (64, 12800),
                  (100, 6400), (200, 4096), (295, 5120)]


@pytest.mark.parametrize("m,k", CLUSTER_SHAPES)
def test_quant_per_token_cluster_rows(pkg, oracle, cuda_dev, m, k):
    x = _x(m, k, seed=m * 11 + k, scale=3.0)
    x[0, k // 3] = 40.0  # absmax in a middle CTA of the cluster
    if m > 2:
        x[2].zero_()  # all-zero row: scale 0, q 0
    q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
    q_ref, s_ref = oracle.quant_per_token(x)
    assert torch.equal(s.cpu(), s_ref) and torch.equal(q.cpu(), q_ref)


@pytest.mark.parametrize("m,i", [(1, 25600), (1, 3200), (8, 12800), (32, 25600), (64, 6400), (150, 4096)])
def test_silu_mul_quant_cluster_rows(pkg, oracle, cuda_dev, m, i):
    gu = _x(m, 2 * i, seed=m + 3 * i, scale=2.0)
    qa, y = pkg.ops.silu_and_mul_quant(gu.to(cuda_dev), with_bf16=True)
    y_ref = oracle.silu_and_mul(gu)
    yc = y.cpu()
    diff = (yc.float() - y_ref.float()).abs()
    assert torch.all(diff <= y_ref.float().abs() * 2.0 ** -7 + 1e-30), float(diff.max())
    q_ref, s_ref = oracle.quant_per_token(yc)
    assert torch.equal(qa.s.cpu(), s_ref) and torch.equal(qa.q.cpu(), q_ref)
    # the quantisation without the bf16 output is the same
    qa2 = pkg.ops.silu_and_mul_quant(gu.to(cuda_dev))
    assert torch.equal(qa2.q.cpu(), qa.q.cpu()) and torch.equal(qa2.s.cpu(), qa.s.cpu())


# Many rows of at most 24 KB: the persistent kernel that keeps several rows in
# flight with bulk copies into shared memory (rows per CTA > pipeline depth,
# ragged last wave, strided rows as in the q slice of a qkv output).
STAGED_SHAPES = [(296, 5120, 5120), (4096, 5120, 5120), (4096, 8192, 10240), (1000, 12288, 12288),
                 (777, 512, 520), (3000, 2048, 2048), (513, 1024, 1536)]


@pytest.mark.parametrize("m,k,ld", STAGED_SHAPES)
def test_quant_per_token_staged_rows(pkg, oracle, cuda_dev, m, k, ld):
    full = _x(m, ld, seed=m + k + ld, scale=2.5)
    full[m // 2, k - 1] = -77.0  # absmax at a row's last element
    full[m - 1].zero_()
    x = full.to(cuda_dev)[:, :k]
    q, s = pkg.ops.quant_per_token(x)
    q_ref, s_ref = oracle.quant_per_token(full[:, :k].contiguous())
    assert torch.equal(s.cpu(), s_ref) and torch.equal(q.cpu(), q_ref)


def test_quant_half_integer_ties(pkg, oracle, cuda_dev):
    """Values whose quotient lies on or within the guard band of a
    half-integer (the rounding path that falls back to the IEEE divide),
    through every quantiser path (register, cluster, staged)."""
    k = 5120
    for m in (1, 64, 600):
        x = torch.zeros(m, k)
        x[:, 0] = 127.0
        ticks = torch.arange(1, k, dtype=torch.float32)
        x[:, 1:] = ((ticks % 254) - 127 + 0.5) * (1 + 1e-6 * (ticks % 7 - 3))
        xb = x.bfloat16()
        q, s = pkg.ops.quant_per_token(xb.to(cuda_dev))
        q_ref, s_ref = oracle.quant_per_token(xb)
        assert torch.equal(s.cpu(), s_ref) and torch.equal(q.cpu(), q_ref), m
