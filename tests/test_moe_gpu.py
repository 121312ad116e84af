"""GPU: the mixture-of-experts W8A8 path (routing layout, quantise-scatter,
grouped tcgen05 GEMMs, top-k sum) against the CPU oracle, stage by stage.

Integer and index stages are bit-exact.  The SiLU*mul product uses the
device's exp (within an ulp of the CPU's), so the stages after it are checked
bit-exact on the kernel's own bf16 product, and the end result against the
pure-CPU chain within the north-star bf16 tolerance."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2


def _weights(oracle, e, h, i, seed):
    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(e, 2 * i, h, generator=g) * 0.02).bfloat16()
    w2 = (torch.randn(e, h, i, generator=g) * 0.02).bfloat16()
    w1q, sw1 = zip(*(oracle.quant_weight_per_channel(w1[x]) for x in range(e)))
    w2q, sw2 = zip(*(oracle.quant_weight_per_channel(w2[x]) for x in range(e)))
    return torch.stack(w1q), torch.stack(sw1), torch.stack(w2q), torch.stack(sw2)


def _routing(oracle, t, e, k, seed, skew=False, drop=False):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(t, e, generator=g)
    if skew:  # most tokens to a few experts: several 128-row blocks per expert
        logits[:, : min(3, e)] += 4.0
    w, ids = oracle.fused_topk(logits, k, renormalize=True)
    if drop and t > 1:
        ids[1, 0] = -1
        ids[t - 1, k - 1] = e  # outside [0, E): dropped too
    return w, ids


def _kernel_silu(pkg, dev):
    """The device's SiLU*mul arithmetic (the bf16-only kernel, which shares it
    with the grouped GEMM's epilogue)."""
    return lambda c1: pkg.ops.silu_and_mul(c1.to(dev)).cpu()


CASES = [
    # (T, H, I, E, topk, skew, drop)
    (1, 256, 128, 8, 2, False, False),        # decode: two experts, one row each
    (5, 512, 384, 8, 2, False, True),         # 3 feature tiles; dropped choices
    (100, 320, 192, 16, 4, False, False),     # partial feature tile (I % 128), N tail in the down GEMM
    (700, 256, 128, 6, 2, True, False),       # several blocks per expert
    (300, 1024, 256, 32, 8, False, True),     # many experts, some empty
    (2048, 256, 128, 64, 8, True, True),      # 16384 slots: the layout kernel spreads over 8 CTAs
]


@pytest.mark.parametrize("t,h,i,e,k,skew,drop", CASES)
def test_moe_stages_bit_exact(pkg, oracle, cuda_dev, t, h, i, e, k, skew, drop):
    ops = pkg.ops
    w1q, sw1, w2q, sw2 = _weights(oracle, e, h, i, seed=t + e)
    topk_w, topk_ids = _routing(oracle, t, e, k, seed=t, skew=skew, drop=drop)
    x = torch.randn(t, h, generator=torch.Generator().manual_seed(7)).bfloat16()
    d = cuda_dev
    ids_d = topk_ids.to(d).contiguous()

    # 1. routing layout
    r = ops.moe_align(ids_d, e)
    torch.cuda.synchronize()
    s_ref, be_ref, inv_ref = oracle.moe_align(topk_ids, e)
    nb = int(r.num_blocks.item())
    assert nb == be_ref.numel() and nb <= r.max_blocks
    assert torch.equal(r.block_expert[:nb].cpu(), be_ref)
    sorted_ids, inv = r.sorted_ids.cpu(), r.inv_pos.cpu()
    assert torch.equal(inv < 0, inv_ref < 0)
    valid = inv >= 0
    slots = torch.arange(inv.numel(), dtype=torch.int32)
    assert torch.equal(sorted_ids[inv[valid].long()], slots[valid])
    # each expert's rows hold the oracle's slots, in any order inside the expert
    for ex in be_ref.unique().tolist():
        blocks = (be_ref == ex).nonzero().flatten()
        lo, hi = int(blocks[0]) * 128, (int(blocks[-1]) + 1) * 128
        assert sorted(sorted_ids[lo:hi].tolist()) == sorted(s_ref[lo:hi].tolist())
    pad = sorted_ids[: nb * 128] == inv.numel()
    assert torch.equal(pad, s_ref == inv.numel())
    assert int(r.sa_sorted[: nb * 128].cpu()[pad].count_nonzero()) == 0

    # 2. quantise into the sorted rows
    q_sorted = ops.moe_quant_scatter(x.to(d), r)
    torch.cuda.synchronize()
    qx, sx = oracle.quant_per_token(x)
    rows = inv[valid].long()
    tok = (slots[valid] // k).long()
    assert torch.equal(q_sorted.cpu()[rows], qx[tok])
    assert torch.equal(r.sa_sorted.cpu()[rows], sx[tok])

    # 3. gate_up grouped GEMM with the SiLU*mul epilogue
    y, amax = ops.moe_gemm(q_sorted, r.sa_sorted, w1q.to(d), sw1.to(d), r, silu=True)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ids_flat = topk_ids.reshape(-1).long()
    c1 = torch.zeros(inv.numel(), 2 * i, dtype=torch.bfloat16)
    for ex in range(e):
        m = (ids_flat == ex) & valid
        if m.any():
            c1[m] = oracle.dequant(oracle.int_gemm(qx[(slots[m] // k).long()], w1q[ex]),
                                   sx[(slots[m] // k).long()], sw1[ex])
    y_dev = pkg.ops.silu_and_mul(c1.to(d)).cpu()            # the device arithmetic on the exact c1
    y_got = y.cpu()[rows]
    assert torch.equal(y_got, y_dev[valid])
    torch.testing.assert_close(y_got.float(), oracle.silu_and_mul(c1)[valid].float(), rtol=RTOL, atol=ATOL)
    am = torch.tensor(amax.cpu()[rows].numpy().view("float32"))
    assert torch.equal(am, y_got.float().abs().amax(dim=1))

    # 4. quantise y (rows in use only)
    qy = ops.moe_quant_rows(y, amax, r)
    torch.cuda.synchronize()
    q2_ref, s2_ref = oracle.quant_per_token(y_got)
    assert torch.equal(qy.q.cpu()[rows], q2_ref)
    assert torch.equal(qy.s.cpu()[rows], s2_ref)

    # 5. down grouped GEMM with the routing weight
    c3 = ops.moe_gemm(qy.q, qy.s, w2q.to(d), sw2.to(d), r, route_w=topk_w.to(d).contiguous())
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ex_v = ids_flat[valid]
    w_v = topk_w.reshape(-1)[valid]
    c3_ref = torch.zeros(rows.numel(), h, dtype=torch.bfloat16)
    for ex in range(e):
        m = ex_v == ex
        if m.any():
            acc = oracle.int_gemm(q2_ref[m], w2q[ex]).to(torch.float32)
            c3_ref[m] = (((acc * s2_ref[m][:, None]) * sw2[ex][None, :]) * w_v[m][:, None]).bfloat16()
    assert torch.equal(c3.cpu()[rows], c3_ref)

    # 6. top-k sum, and the whole chain through the one-call entry
    out = ops.moe_sum(c3, r)
    want, _ = oracle.moe_experts_w8a8(x, w1q, sw1, w2q, sw2, topk_w, topk_ids, silu_y=_kernel_silu(pkg, d))
    assert torch.equal(out.cpu(), want)
    full = ops.fused_experts_w8a8(x.to(d), w1q.to(d), sw1.to(d), w2q.to(d), sw2.to(d), topk_w.to(d), ids_d)
    assert torch.equal(full.cpu(), want)
    cpu_chain, _ = oracle.moe_experts_w8a8(x, w1q, sw1, w2q, sw2, topk_w, topk_ids)
    torch.testing.assert_close(full.cpu().float(), cpu_chain.float(), rtol=RTOL, atol=ATOL)


def test_moe_empty_batch_and_graph_capture(pkg, oracle, cuda_dev):
    ops = pkg.ops
    e, h, i, k = 8, 256, 128, 2
    w1q, sw1, w2q, sw2 = [t.to(cuda_dev) for t in _weights(oracle, e, h, i, seed=3)]
    x0 = torch.empty(0, h, dtype=torch.bfloat16, device=cuda_dev)
    ids0 = torch.empty(0, k, dtype=torch.int32, device=cuda_dev)
    out0 = ops.fused_experts_w8a8(x0, w1q, sw1, w2q, sw2, torch.empty(0, k, device=cuda_dev), ids0)
    assert tuple(out0.shape) == (0, h)
    # capture the six launches in a CUDA graph; replays match the eager call
    t = 64
    topk_w, topk_ids = _routing(oracle, t, e, k, seed=5)
    x = torch.randn(t, h, generator=torch.Generator().manual_seed(9)).bfloat16().to(cuda_dev)
    wd, idd = topk_w.to(cuda_dev).contiguous(), topk_ids.to(cuda_dev).contiguous()
    eager = ops.fused_experts_w8a8(x, w1q, sw1, w2q, sw2, wd, idd)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.fused_experts_w8a8(x, w1q, sw1, w2q, sw2, wd, idd)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        captured = ops.fused_experts_w8a8(x, w1q, sw1, w2q, sw2, wd, idd)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, eager)
    assert ops.device_error() == 0


def test_moe_layer_forward(pkg, oracle, cuda_dev):
    pkg.reset_tp_info()
    pkg.set_tp_info(0, 1)
    pkg.DistributedCommunicator.plugins = [pkg.distributed.TorchDistributedImpl()]
    try:
        e, h, i, k, t = 16, 512, 256, 4, 77
        layer = pkg.MoELayer(num_experts=e, top_k=k, hidden_size=h, intermediate_size=i)
        w1q, sw1, w2q, sw2 = _weights(oracle, e, h, i, seed=11)
        layer.load_state_dict({"gate_up_proj": w1q.to(cuda_dev), "gate_up_proj_scale": sw1.to(cuda_dev),
                               "down_proj": w2q.to(cuda_dev), "down_proj_scale": sw2.to(cuda_dev)})
        g = torch.Generator().manual_seed(12)
        x = torch.randn(t, h, generator=g).bfloat16()
        logits = torch.randn(t, e, generator=g)
        y = layer.forward(x.to(cuda_dev), logits.to(cuda_dev))
        w_dev, ids_dev = layer.route(logits.to(cuda_dev))
        w_ref, ids_ref = oracle.fused_topk(logits, k, renormalize=True)
        assert torch.equal(ids_dev.cpu(), ids_ref)
        torch.testing.assert_close(w_dev.cpu(), w_ref, rtol=1e-5, atol=1e-6)
        want, _ = oracle.moe_experts_w8a8(x, w1q, sw1, w2q, sw2, w_dev.cpu(), ids_dev.cpu(),
                                          silu_y=_kernel_silu(pkg, cuda_dev))
        assert torch.equal(y.cpu(), want)
    finally:
        pkg.reset_tp_info()
