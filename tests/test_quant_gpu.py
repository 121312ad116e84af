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


# Many rows of at most 16384 values: the persistent warp-group kernel (1, 2
# or 4 warps per row held in registers; rows per group > 1, ragged last wave,
# rows that do not fill every lane, strided rows as in the q slice of a qkv
# output).
STAGED_SHAPES = [(296, 5120, 5120), (4096, 5120, 5120), (4096, 8192, 10240), (1000, 12288, 12288),
                 (777, 512, 520), (3000, 2048, 2048), (513, 1024, 1536), (400, 16384, 16384), (350, 40, 40),
                 (9000, 3584, 3584)]


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


# Many SiLU*mul rows (one CTA per row: in registers up to 8192 outputs, staged
# in shared memory beyond), strided, with an all-zero product row and the
# absmax at a row's last element.
SILU_MANY = [(296, 25600), (700, 12800), (300, 12288), (4096, 3200), (500, 6400), (777, 1000), (1200, 8192),
             (2000, 25600)]


@pytest.mark.parametrize("m,i", SILU_MANY)
def test_silu_mul_quant_many_rows(pkg, oracle, cuda_dev, m, i):
    gu = _x(m, 2 * i + 8, seed=m * 5 + i, scale=2.0)[:, : 2 * i]  # strided rows
    gu[m // 3, i - 1] = 30.0  # a large product at a row's last element
    gu[m // 3, 2 * i - 1] = 4.0
    gu[m - 1, i:] = 0  # all-zero product row
    gd = gu.to(cuda_dev)
    qa, y = pkg.ops.silu_and_mul_quant(gd, with_bf16=True)
    y_ref = oracle.silu_and_mul(gu.contiguous())
    yc = y.cpu()
    diff = (yc.float() - y_ref.float()).abs()
    assert torch.all(diff <= y_ref.float().abs() * 2.0 ** -7 + 1e-30), float(diff.max())
    assert (yc != y_ref).float().mean().item() < 1e-3
    q_ref, s_ref = oracle.quant_per_token(yc)
    assert torch.equal(qa.s.cpu(), s_ref) and torch.equal(qa.q.cpu(), q_ref)
    assert float(qa.s[m - 1]) == 0.0
    qa2 = pkg.ops.silu_and_mul_quant(gd)
    assert torch.equal(qa2.q.cpu(), qa.q.cpu()) and torch.equal(qa2.s.cpu(), qa.s.cpu())


def _all_bf16_upto(amax: float) -> torch.Tensor:
    """Every finite bf16 value v with |v| <= amax (both signs), amax first."""
    bits = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    a = torch.tensor(amax).bfloat16()
    pos = bits[bits.float() <= a.float()]
    return torch.cat([a.reshape(1), pos, -pos])


@pytest.mark.parametrize("many", [False, True])
def test_quant_every_bf16_value(pkg, oracle, cuda_dev, many):
    """For absmax values across the whole exponent range (subnormal scales
    included: 1/s is infinite below s = 2^-128), every bf16 value that can
    share a row with that absmax is quantised bit-exactly.  Rows of 16384
    values, each led by its absmax: 18 rows reach the cluster kernel, the
    same rows repeated to >= 296 the warp-group kernel."""
    width = 16384
    rows = []
    for amax in (1.0, 3.140625, 127.0, 1e-20, 2.0e-36, 1.2e-38, 5.0e-39, 1.0e-39, 9.2e-41, 3.0e38):
        v = _all_bf16_upto(amax)
        n = (v.numel() + width - 2) // (width - 1)
        pad = torch.zeros(n * (width - 1) - (v.numel() - 1), dtype=torch.bfloat16)
        body = torch.cat([v[1:], pad]).reshape(n, width - 1)
        rows.append(torch.cat([v[:1].expand(n, 1), body], dim=1))
    x = torch.cat(rows)
    if many:
        x = x.repeat((296 + x.shape[0] - 1) // x.shape[0], 1)
    q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
    q_ref, s_ref = oracle.quant_per_token(x)
    assert torch.equal(s.cpu(), s_ref)
    bad = (q.cpu() != q_ref).nonzero()
    assert bad.numel() == 0, (bad[:5].tolist(), x[bad[0, 0], bad[0, 1]].item() if bad.numel() else None)


def test_quant_subnormal_scale_rows(pkg, oracle, cuda_dev):
    """Rows whose scale is subnormal (absmax below ~1.5e-36): through the
    warp-group, cluster and register paths, and from the fused SiLU*mul."""
    for m, k in ((400, 5120), (3, 5120), (2, 256)):
        x = _x(m, k, seed=m + k)
        for r, amax in enumerate((1.0e-38, 9.2e-41, 3.0e-39)):
            if r < m:
                x[r] = (x[r].float() / x[r].float().abs().max() * amax).bfloat16()
        q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
        q_ref, s_ref = oracle.quant_per_token(x)
        assert torch.equal(s.cpu(), s_ref) and torch.equal(q.cpu(), q_ref)
        assert int(q[0].abs().max()) == 127
    gu = _x(300, 2 * 3200, seed=5)
    gu[:, 3200:] = (gu[:, 3200:].float() * 1e-38).bfloat16()
    qa, y = pkg.ops.silu_and_mul_quant(gu.to(cuda_dev), with_bf16=True)
    q_ref, s_ref = oracle.quant_per_token(y.cpu())
    assert torch.equal(qa.s.cpu(), s_ref) and torch.equal(qa.q.cpu(), q_ref)
