"""GPU: fused RMSNorm + per-token quant (``w8a8_rmsnorm_quant``) against the
CPU oracle (``rmsnorm`` / ``rmsnorm_quant``, following M/layers/norm.py:8-38).

* residual_out = bf16(x + residual): bit-exact.
* the bf16 normalised rows: within one bf16 ulp of the oracle, and at most
  0.1 % of elements differ (the fp32 sum of squares runs in another order on
  the GPU; the sqrt and divide are correctly rounded on both sides).
* int8 values and scales: bit-exact against the oracle's quantisation of the
  kernel's own normalised rows; against the oracle's whole chain, q within one
  step on at most 0.1 % of elements.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _data(m, k, seed, residual):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).bfloat16()
    w = (1.0 + 0.1 * torch.randn(k, generator=g)).bfloat16()
    r = torch.randn(m, k, generator=g).bfloat16() if residual else None
    return x, w, r


def _ulp_diff(a, b):
    ai = a.view(torch.int16).int()
    bi = b.view(torch.int16).int()
    return (ai - bi).abs()


# one CTA per row below 2 x 148 rows; warp groups (1, 2 or 4 warps per row,
# persistent grid) from there on
@pytest.mark.parametrize("m,k,residual", [(1, 1024, False), (7, 4096, True), (256, 5120, True),
                                          (33, 8192, False), (100, 2048, True), (5, 24, True),
                                          (300, 5120, True), (4096, 5120, True), (1000, 8192, False),
                                          (600, 2048, True), (777, 256, False), (300, 64, True)])
def test_rmsnorm_quant_matches_oracle(pkg, oracle, cuda_dev, m, k, residual):
    x, w, r = _data(m, k, m * 31 + k, residual)
    qw, sw, yw, resw = oracle.rmsnorm_quant(x, w, EPS, r)
    xd, wd = x.to(cuda_dev), w.to(cuda_dev)
    rd = r.to(cuda_dev) if residual else None
    qa, res, y = pkg.ops.rmsnorm_quant(xd, wd, EPS, rd, with_bf16=True)
    torch.cuda.synchronize()
    if residual:
        assert res is rd and torch.equal(res.cpu(), resw)   # updated in place, bit-exact
    else:
        assert res is xd
    d = _ulp_diff(y.cpu(), yw)
    assert int(d.max()) <= 1
    assert float((d > 0).float().mean()) <= 1e-3
    q2, s2 = oracle.quant_per_token(y.cpu())
    assert torch.equal(qa.q.cpu(), q2) and torch.equal(qa.s.cpu(), s2)
    # against the oracle's own chain: a row's normalised value one bf16 ulp
    # away can cross a quantisation rounding boundary, so q may move by one step
    dq = (qa.q.cpu().int() - qw.int()).abs()
    assert int(dq.max()) <= 1 and float((dq > 0).float().mean()) <= 1e-3
    torch.testing.assert_close(qa.s.cpu(), sw, atol=0, rtol=2 ** -7)


def test_zero_rows_and_layer_chain(pkg, oracle, cuda_dev):
    """An all-zero row gives q = 0, s = 0; the layer feeds qkv directly."""
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(0, 1)
    try:
        hidden, hd, nq, nkv = 256, 32, 4, 2
        x, w, r = _data(9, hidden, 7, True)
        x[3] = 0
        r[3] = 0
        norm = pkg.RMSNormFusedQuant(hidden, EPS)
        norm.load_state_dict({"weight": w.to(cuda_dev)})
        g = torch.Generator().manual_seed(2)
        wq, ws = oracle.quant_weight_per_channel((torch.randn((nq + 2 * nkv) * hd, hidden, generator=g) * 0.05)
                                                 .bfloat16())
        qkv = pkg.LinearQKVMerged(hidden, hd, nq, nkv, has_bias=False)
        qkv.load_state_dict({"weight": wq.to(cuda_dev), "weight_scale": ws.to(cuda_dev)})
        rd = r.to(cuda_dev)
        qa, res = norm.forward(x.to(cuda_dev), rd)
        assert res is rd
        assert int(qa.q[3].abs().max()) == 0 and float(qa.s[3]) == 0.0
        out = qkv.forward(qa)
        qw_, sw_, _, _ = oracle.rmsnorm_quant(x, w, EPS, r)
        want = oracle.dequant(oracle.int_gemm(qw_, wq), sw_, ws)
        torch.testing.assert_close(out.cpu().float(), want.float(), atol=1e-2, rtol=1e-2)
    finally:
        D.reset_tp_info()


def test_rmsnorm_quant_rejects_bad_arguments(pkg, cuda_dev):
    x = torch.zeros(4, 16, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(pkg.W8A8Error):
        pkg.ops.rmsnorm_quant(x, torch.ones(8, dtype=torch.bfloat16, device=cuda_dev), EPS)
    big = torch.zeros(2, 16384, dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(pkg.W8A8Error, match="8192"):
        pkg.ops.rmsnorm_quant(big, torch.ones(16384, dtype=torch.bfloat16, device=cuda_dev), EPS)
