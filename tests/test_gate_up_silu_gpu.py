"""GPU: the gate_up GEMM with SiLU*mul in its epilogue (w8a8_gemm_silu) and
the quantiser with a known row absmax (w8a8_quant_rows_amax) against the
two-step path they replace -- gate_up GEMM, then the fused SiLU*mul
quantiser -- bit for bit (bf16 product, int8 values, fp32 scales), and that
path against the CPU oracle."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(m, n2, k, seed, bias, dev, O):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).bfloat16()
    w = (torch.randn(n2, k, generator=g) * 0.05).bfloat16()
    wq, ws = O.quant_weight_per_channel(w)
    xq, xs = O.quant_per_token(x)
    b = (torch.randn(n2, generator=g) * 0.1).bfloat16() if bias else None
    to = lambda t: None if t is None else t.to(dev)  # noqa: E731
    return xq, xs, wq, ws, b, (to(xq), to(wq), to(xs), to(ws), to(b))


@pytest.mark.parametrize("m,n2,k,bias", [(4096, 51200, 5120, False), (300, 2048, 1024, True),
                                         (777, 24576, 4096, False), (129, 512, 256, True),
                                         (2048, 7168, 8192, False)])
def test_gate_up_silu_matches_two_step(pkg, oracle, cuda_dev, m, n2, k, bias):
    ops = pkg.ops
    xq, xs, wq, ws, b, (aq, wq_d, sa, sw, bd) = _case(m, n2, k, m + n2, bias, cuda_dev, oracle)
    fused = ops.gate_up_silu_quant(aq, wq_d, sa, sw, bd, with_bf16=True)
    assert fused is not None, "the fused path should apply at this shape"
    qa, y = fused
    gu = ops.w8a8_gemm(aq, wq_d, sa, sw, bd)
    ref, y_ref = ops.silu_and_mul_quant(gu, with_bf16=True)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), y_ref.cpu())
    assert torch.equal(qa.s.cpu(), ref.s.cpu())
    assert torch.equal(qa.q.cpu(), ref.q.cpu())
    # the gate_up GEMM against the oracle (bit-exact), the SiLU*mul product
    # within one bf16 ulp of the CPU's, and its quantisation bit-exact
    if m * n2 <= 1 << 24:
        gu_ref = oracle.dequant(oracle.int_gemm(xq, wq), xs, ws, b)
        assert torch.equal(gu.cpu(), gu_ref)
        y_o = oracle.silu_and_mul(gu_ref)
        diff = (y.cpu().float() - y_o.float()).abs()
        assert torch.all(diff <= y_o.float().abs() * 2.0 ** -7 + 1e-30)
    q_o, s_o = oracle.quant_per_token(y.cpu())
    assert torch.equal(qa.q.cpu(), q_o) and torch.equal(qa.s.cpu(), s_o)


def test_gate_up_silu_declines_outside_its_range(pkg, oracle, cuda_dev):
    """M <= 128, or 2I not a multiple of 256: None, and the layer's
    forward_silu_quant takes the two-step path with the same result."""
    ops = pkg.ops
    for m, n2, k in ((64, 512, 256), (300, 2 * 200, 256)):
        _, _, _, _, _, (aq, wq_d, sa, sw, _) = _case(m, n2, k, 7, False, cuda_dev, oracle)
        assert ops.gate_up_silu_quant(aq, wq_d, sa, sw) is None


def test_layer_forward_silu_quant(pkg, oracle, cuda_dev):
    """LinearColParallelMerged.forward_silu_quant == silu_and_mul_quant(forward)."""
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(0, 1)
    for m in (50, 1000):
        layer = pkg.LinearColParallelMerged(1024, [1536, 1536], has_bias=False)
        g = torch.Generator().manual_seed(m)
        w = (torch.randn(3072, 1024, generator=g) * 0.05).bfloat16()
        wq, ws = oracle.quant_weight_per_channel(w)
        layer.load_state_dict({"weight": wq.to(cuda_dev), "weight_scale": ws.to(cuda_dev)})
        x = torch.randn(m, 1024, generator=g).bfloat16().to(cuda_dev)
        a = layer.forward_silu_quant(x)
        b = pkg.ops.silu_and_mul_quant(layer.forward(x))
        torch.cuda.synchronize()
        assert torch.equal(a.q.cpu(), b.q.cpu()) and torch.equal(a.s.cpu(), b.s.cpu())
    D.reset_tp_info()
