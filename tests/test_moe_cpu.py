"""CPU: the mixture-of-experts restatement (oracle) pinned to the reference's
own example and cross-checked slot by slot; host validation of the MoE C
entry points (no GPU calls)."""
from __future__ import annotations

import pytest
import torch


def test_align_matches_the_reference_docstring_example(oracle):
    # moe_align_block_size's worked example (M/moe/fused.py:52-71): block 4,
    # expert ids 1..4 (bucket 0 unused), 12 slots
    ids = torch.tensor([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], dtype=torch.int32)
    sorted_ids, block_expert, row_of_slot = oracle.moe_align(ids, 5, block=4)
    assert sorted_ids.tolist() == [3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12]
    assert block_expert.tolist() == [1, 2, 3, 4]
    for s, r in enumerate(row_of_slot.tolist()):
        assert sorted_ids[r] == s


def test_align_drops_ids_outside_the_expert_range(oracle):
    ids = torch.tensor([[0, -1], [3, 7], [0, 0]], dtype=torch.int32)
    sorted_ids, block_expert, row_of_slot = oracle.moe_align(ids, 4, block=128)
    assert block_expert.tolist() == [0, 3]
    assert row_of_slot.tolist() == [0, -1, 128, -1, 1, 2]
    assert sorted_ids[:3].tolist() == [0, 4, 5] and int(sorted_ids[3]) == 6


def test_fused_topk_renormalises_twice(oracle):
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(7, 16, generator=g)
    w, ids = oracle.fused_topk(logits, 4, renormalize=True)
    p = torch.softmax(logits, dim=-1)
    want_ids = torch.topk(p, 4, dim=-1).indices
    assert torch.equal(ids.long(), want_ids)
    s = w.sum(-1)
    assert torch.allclose(s, torch.ones_like(s), atol=1e-6)
    w0, _ = oracle.fused_topk(logits, 4, renormalize=False)
    assert torch.allclose(w0, torch.gather(p, 1, want_ids))


def _moe_weights(oracle, e, h, i, seed):
    g = torch.Generator().manual_seed(seed)
    w1 = (torch.randn(e, 2 * i, h, generator=g) * 0.02).bfloat16()
    w2 = (torch.randn(e, h, i, generator=g) * 0.02).bfloat16()
    w1q, sw1 = zip(*(oracle.quant_weight_per_channel(w1[x]) for x in range(e)))
    w2q, sw2 = zip(*(oracle.quant_weight_per_channel(w2[x]) for x in range(e)))
    return torch.stack(w1q), torch.stack(sw1), torch.stack(w2q), torch.stack(sw2)


def test_moe_restatement_matches_a_per_slot_loop(oracle):
    """The per-expert vectorised restatement equals a literal per-(token,
    choice) loop over the dense W8A8 linear oracle."""
    t, h, i, e, k = 9, 64, 48, 6, 3
    w1q, sw1, w2q, sw2 = _moe_weights(oracle, e, h, i, seed=1)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(t, h, generator=g).bfloat16()
    w, ids = oracle.fused_topk(torch.randn(t, e, generator=g), k, renormalize=True)
    ids[2, 1] = -1  # a dropped choice
    out, parts = oracle.moe_experts_w8a8(x, w1q, sw1, w2q, sw2, w, ids)
    want = torch.zeros(t, h, dtype=torch.float32)
    for tt in range(t):
        for j in range(k):
            ex = int(ids[tt, j])
            if ex < 0:
                continue
            c1 = oracle.w8a8_linear(x[tt:tt + 1], w1q[ex], sw1[ex])[3]
            q2, s2, _ = oracle.silu_mul_quant(c1)
            acc = oracle.int_gemm_int64(q2, w2q[ex]).to(torch.float32)
            c3 = (((acc * s2[:, None]) * sw2[ex][None, :]) * w[tt, j]).bfloat16()
            assert torch.equal(parts["c3"][tt, j], c3[0])
            want[tt] = want[tt] + c3[0].float()
    assert torch.equal(out, want.bfloat16())


def test_moe_host_validation(pkg):
    lib = pkg.load_library()
    L = pkg._lib
    assert lib.w8a8_moe_max_blocks(0, 8) == 0
    assert lib.w8a8_moe_max_blocks(32768, 128) == (32768 + 127 * 128) // 128
    assert lib.w8a8_moe_max_blocks(3, 64) == 3            # at most one block per slot
    assert lib.w8a8_moe_align(16, 8, 2048, 16, 16, 16, 16, 16, None) == L.ERR_UNSUPPORTED
    assert b"experts" in lib.w8a8_last_error()
    assert lib.w8a8_moe_align(16, 8, 8, None, 16, 16, 16, 16, None) == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_quant_scatter(16, 64, 4, 64, 16, 0, 16, 16, None) == L.ERR_UNSUPPORTED
    assert lib.w8a8_moe_quant_scatter(16, 64, 4, 60, 16, 2, 16, 16, None) == L.ERR_INVALID_ARG
    # grouped GEMM: null operand, K % 16, SiLU with N % 32, routing weight without sorted ids
    assert lib.w8a8_moe_gemm(None, 16, 16, 16, 16, 16, 4, 16, None, 64, 16, None, 8, 256, 128, None) \
        == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_gemm(16, 16, 16, 16, 16, 16, 4, 16, None, 64, 16, None, 8, 256, 120, None) \
        == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_gemm(16, 16, 16, 16, 16, 16, 4, 16, None, 64, 16, 16, 8, 272, 128, None) \
        == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_gemm(16, 16, 16, 16, 16, 16, 4, None, 16, 64, 16, None, 8, 256, 128, None) \
        == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_gemm(16, 16, 16, 16, 16, 16, 4, 16, 16, 64, 16, 16, 8, 256, 128, None) \
        == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_gemm(16, 24, 16, 16, 16, 16, 4, 16, None, 64, 16, None, 8, 256, 128, None) \
        == L.ERR_ALIGNMENT
    assert lib.w8a8_moe_quant_rows(16, 64, 16, 16, 16, None, 4, 64, None) == L.ERR_INVALID_ARG
    assert lib.w8a8_moe_sum(16, 64, 16, 4, 0, 64, 16, 64, None) == L.ERR_UNSUPPORTED
    assert lib.w8a8_moe_sum(16, 64, 16, 4, 2, 60, 16, 64, None) == L.ERR_INVALID_ARG
    # empty batches are no-ops
    assert lib.w8a8_moe_sum(None, 64, None, 0, 2, 64, None, 64, None) == L.OK
    assert lib.w8a8_moe_gemm(None, None, None, None, None, None, 0, None, None, 0, None, None, 8, 256, 128, None) \
        == L.OK


def test_moe_layer_state_dict_contract(pkg):
    pkg.reset_tp_info()
    pkg.set_tp_info(0, 1)
    try:
        layer = pkg.MoELayer(num_experts=4, top_k=2, hidden_size=64, intermediate_size=32)
        sd = layer.state_dict()
        assert sorted(sd) == ["down_proj", "down_proj_scale", "gate_up_proj", "gate_up_proj_scale"]
        assert tuple(sd["gate_up_proj"].shape) == (4, 64, 64) and sd["gate_up_proj"].dtype == torch.int8
        assert tuple(sd["down_proj"].shape) == (4, 64, 32) and tuple(sd["down_proj_scale"].shape) == (4, 64)
        with pytest.raises(ValueError):
            pkg.MoELayer(4, 2, 64, 32, activation="gelu")
        with pytest.raises(pkg.W8A8Error):
            pkg.ops.fused_experts_w8a8(torch.zeros(2, 64, dtype=torch.bfloat16), sd["gate_up_proj"],
                                       sd["gate_up_proj_scale"], sd["down_proj"], sd["down_proj_scale"],
                                       torch.zeros(2, 2), torch.zeros(2, 2, dtype=torch.int32))
    finally:
        pkg.reset_tp_info()


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_loader_shards_feed_the_tp_experts(pkg, oracle, tp):
    """Per-rank expert tensors from the loader (HF per-expert layout in) are
    exactly the intermediate-dim shards the TP restatement uses, and
    MoELayer's state dict at that TP accepts them."""
    E, H, I, T, K = 4, 64, 64, 6, 2
    g = torch.Generator().manual_seed(9)
    p = "model.layers.0.mlp."
    items, w1, w2 = [], [], []
    for e in range(E):
        gate = (torch.randn(I, H, generator=g) * 0.02).bfloat16()
        up = (torch.randn(I, H, generator=g) * 0.02).bfloat16()
        down = (torch.randn(H, I, generator=g) * 0.02).bfloat16()
        items += [(f"{p}experts.{e}.gate_proj.weight", gate), (f"{p}experts.{e}.up_proj.weight", up),
                  (f"{p}experts.{e}.down_proj.weight", down)]
        w1.append(torch.cat([gate, up]))
        w2.append(down)
    q1 = [oracle.quant_weight_per_channel(w) for w in w1]
    q2 = [oracle.quant_weight_per_channel(w) for w in w2]
    w1q, sw1 = torch.stack([q for q, _ in q1]), torch.stack([s for _, s in q1])
    w2q, sw2 = torch.stack([q for q, _ in q2]), torch.stack([s for _, s in q2])
    x = torch.randn(T, H, generator=g).bfloat16()
    tw, tid = oracle.fused_topk(torch.randn(T, E, generator=g), K, renormalize=True)
    want, parts = oracle.tp_moe_experts(x, w1q, sw1, w2q, sw2, tw, tid, tp)
    got_parts = []
    for r in range(tp):
        sd = pkg.load_w8a8_state_dict(items, r, tp, None, quantise=oracle.quant_weight_per_channel, num_experts=E)
        pre = p + "experts."
        out, _ = oracle.moe_experts_w8a8(x, sd[pre + "gate_up_proj"], sd[pre + "gate_up_proj_scale"],
                                         sd[pre + "down_proj"], sd[pre + "down_proj_scale"], tw, tid)
        got_parts.append(out)
        assert torch.equal(out, parts[r])
        pkg.reset_tp_info()
        pkg.set_tp_info(r, tp)
        try:
            layer = pkg.MoELayer(num_experts=E, top_k=K, hidden_size=H, intermediate_size=I)
            layer.load_state_dict({k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)})
            assert tuple(layer.gate_up_proj.shape) == (E, 2 * I // tp, H)
        finally:
            pkg.reset_tp_info()
    assert torch.equal(oracle.all_reduce_sum(got_parts) if tp > 1 else got_parts[0], want)
    if tp == 1:
        assert torch.equal(want, oracle.moe_experts_w8a8(x, w1q, sw1, w2q, sw2, tw, tid)[0])


@pytest.mark.parametrize("renorm", [True, False])
def test_layer_routing_follows_fused_topk(pkg, oracle, renorm):
    """MoELayer.route (torch ops, run here on CPU tensors) is fused_topk's
    arithmetic: the same experts and the same weights."""
    pkg.reset_tp_info()
    pkg.set_tp_info(0, 1)
    try:
        layer = pkg.MoELayer(num_experts=16, top_k=4, hidden_size=64, intermediate_size=32, renormalize=renorm)
        logits = torch.randn(33, 16, generator=torch.Generator().manual_seed(4))
        w, ids = layer.route(logits)
        w_ref, ids_ref = oracle.fused_topk(logits, 4, renormalize=renorm)
        assert ids.dtype == torch.int32 and w.dtype == torch.float32
        assert torch.equal(ids, ids_ref) and torch.equal(w, w_ref)
    finally:
        pkg.reset_tp_info()
