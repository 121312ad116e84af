"""CPU: W8A8 checkpoint loading (``weights.py``).

* Sharding is pinned to the reference's own ``_shard_tensor`` outputs
  (``tests/golden/shard_layout.pt``, generated from M/models/weight.py:34-52).
* Quantise-at-load of a bf16 checkpoint gives, for every rank, exactly the
  shards the oracle builds (per-channel quantisation of the UNSHARDED weight,
  positional shard, scales replicated on row-parallel splits, q|k|v and
  gate|up merged in slot order) -- the quantiser is injected (the oracle's
  rule) so the stream logic is tested without a GPU.
* An int8 checkpoint (weight + weight_scale) passes through to the same
  state dict, without any quantisation.
* The result loads into the W8A8 layer classes at every TP size.
"""
from __future__ import annotations

import pytest
import torch

from conftest import golden

HIDDEN, NQ, NKV, HD, INTER, VOCAB = 64, 8, 2, 8, 96, 100


def _checkpoint(seed: int = 0, layers: int = 2):
    """HF-style tensors of a small Qwen2-like model (q/k/v biases)."""
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, scale=0.02):
        return (torch.randn(*shape, generator=g) * scale).bfloat16()

    items = [("model.embed_tokens.weight", rnd(VOCAB, HIDDEN, scale=1.0))]
    for i in range(layers):
        p = f"model.layers.{i}."
        items += [
            (p + "input_layernorm.weight", rnd(HIDDEN, scale=1.0)),
            (p + "self_attn.q_proj.weight", rnd(NQ * HD, HIDDEN)),
            (p + "self_attn.q_proj.bias", rnd(NQ * HD, scale=0.1)),
            (p + "self_attn.k_proj.weight", rnd(NKV * HD, HIDDEN)),
            (p + "self_attn.k_proj.bias", rnd(NKV * HD, scale=0.1)),
            (p + "self_attn.v_proj.weight", rnd(NKV * HD, HIDDEN)),
            (p + "self_attn.v_proj.bias", rnd(NKV * HD, scale=0.1)),
            (p + "self_attn.o_proj.weight", rnd(HIDDEN, NQ * HD)),
            (p + "post_attention_layernorm.weight", rnd(HIDDEN, scale=1.0)),
            (p + "mlp.gate_proj.weight", rnd(INTER, HIDDEN)),
            (p + "mlp.up_proj.weight", rnd(INTER, HIDDEN)),
            (p + "mlp.down_proj.weight", rnd(HIDDEN, INTER)),
        ]
    items += [("model.norm.weight", rnd(HIDDEN, scale=1.0)), ("lm_head.weight", rnd(VOCAB, HIDDEN))]
    return items


def _expected(oracle, items, r, n):
    """The oracle's state dict for rank r of n."""
    full = dict(items)
    out = {}
    layers = sorted({k.split(".")[2] for k in full if k.startswith("model.layers.")})
    for i in layers:
        p = f"model.layers.{i}."
        for fused, parts in (("self_attn.qkv_proj", ("q", "k", "v")), ("mlp.gate_up_proj", ("gate", "up"))):
            base = "self_attn." if fused.startswith("self_attn") else "mlp."
            ws, ss, bs = [], [], []
            for part in parts:
                key = p + base + f"{part}_proj.weight"
                q, s = oracle.quant_weight_per_channel(full[key])
                ws.append(oracle.shard_tensor(key, q, r, n, NKV))
                ss.append(oracle.shard_scale(key, s, r, n, NKV))
                bkey = p + base + f"{part}_proj.bias"
                if bkey in full:
                    bs.append(oracle.shard_tensor(bkey, full[bkey], r, n, NKV))
            out[p + fused + ".weight"] = torch.cat(ws)
            out[p + fused + ".weight_scale"] = torch.cat(ss)
            if bs:
                out[p + fused + ".bias"] = torch.cat(bs)
        for row in ("self_attn.o_proj", "mlp.down_proj"):
            key = p + row + ".weight"
            q, s = oracle.quant_weight_per_channel(full[key])
            out[key] = oracle.shard_tensor(key, q, r, n, NKV)
            out[key + "_scale"] = oracle.shard_scale(key, s, r, n, NKV)
        for norm in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            out[p + norm] = full[p + norm]
    per = -(-VOCAB // n)
    for key in ("model.embed_tokens.weight", "lm_head.weight"):
        out[key] = full[key][r * per:min((r + 1) * per, VOCAB)]
    out["model.norm.weight"] = full["model.norm.weight"]
    return out


def _assert_same(got, want):
    assert sorted(got) == sorted(want)
    for k in want:
        assert got[k].dtype == want[k].dtype, k
        assert torch.equal(got[k], want[k]), k


def test_shard_tensor_matches_reference_goldens(pkg):
    g = golden("shard_layout.pt")
    for key, ref in g["shards"].items():
        name, r, n = key.split("|")
        got = pkg.weights.shard_tensor(name, g["inputs"][name], int(r), int(n), g["num_kv_heads"])
        assert torch.equal(got, ref), key


@pytest.mark.parametrize("world", [1, 2, 4])
def test_quantise_at_load_matches_oracle(pkg, oracle, world):
    items = _checkpoint()
    for r in range(world):
        got = pkg.load_w8a8_state_dict(items, r, world, NKV, quantise=oracle.quant_weight_per_channel)
        _assert_same(got, _expected(oracle, items, r, world))
        # row-parallel shards keep the whole scale vector; kv heads replicate at world 4
        assert got["model.layers.0.self_attn.o_proj.weight_scale"].shape == (HIDDEN,)
        assert got["model.layers.0.self_attn.qkv_proj.weight"].dtype == torch.int8


def test_int8_checkpoint_passes_through(pkg, oracle):
    items = _checkpoint(seed=3)
    quantised = []
    for name, t in items:
        if pkg.weights.is_linear_weight(name):
            q, s = oracle.quant_weight_per_channel(t)
            quantised += [(name, q), (name + "_scale", s)]
        else:
            quantised.append((name, t))

    def refuse(_w):
        raise AssertionError("an int8 checkpoint must not be quantised again")

    for world in (1, 2, 4):
        for r in range(world):
            got = pkg.load_w8a8_state_dict(quantised, r, world, NKV, quantise=refuse)
            _assert_same(got, _expected(oracle, items, r, world))


@pytest.mark.parametrize("world", [1, 2, 4])
def test_state_dict_loads_into_layers(pkg, oracle, world):
    D = pkg.distributed
    items = _checkpoint(seed=5, layers=1)
    try:
        for r in range(world):
            D.reset_tp_info()
            D.set_tp_info(r, world)
            sd = pkg.load_w8a8_state_dict(items, r, world, NKV, quantise=oracle.quant_weight_per_channel)
            mods = {
                "model.layers.0.self_attn.qkv_proj": pkg.LinearQKVMerged(HIDDEN, HD, NQ, NKV, has_bias=True),
                "model.layers.0.self_attn.o_proj": pkg.LinearOProj(NQ * HD, HIDDEN, has_bias=False),
                "model.layers.0.mlp": pkg.GatedMLP(HIDDEN, INTER),
            }
            for prefix, mod in mods.items():
                sub = {k: v for k, v in sd.items() if k.startswith(prefix + ".")}
                mod.load_state_dict(sub, prefix=prefix)
            assert mods["model.layers.0.mlp"].down_proj.weight.shape == (HIDDEN, INTER // world)
            assert mods["model.layers.0.self_attn.qkv_proj"].weight.dtype == torch.int8
    finally:
        D.reset_tp_info()


def test_incomplete_merge_group_raises(pkg, oracle):
    items = [(k, v) for k, v in _checkpoint(layers=1) if ".v_proj." not in k]
    with pytest.raises(pkg.W8A8Error, match="incomplete merge"):
        pkg.load_w8a8_state_dict(items, 0, 2, NKV, quantise=oracle.quant_weight_per_channel)


def test_prefixes_and_skipped_towers(pkg, oracle):
    items = [("language_model." + k, v) for k, v in _checkpoint(layers=1)]
    items.append(("vision_tower.blocks.0.attn.q_proj.weight", torch.zeros(4, 4, dtype=torch.bfloat16)))
    got = pkg.load_w8a8_state_dict(items, 0, 1, NKV, quantise=oracle.quant_weight_per_channel)
    assert not any(k.startswith(("language_model.", "vision_tower.")) for k in got)
    _assert_same(got, _expected(oracle, _checkpoint(layers=1), 0, 1))


def test_scales_must_be_vectors(pkg):
    with pytest.raises(pkg.W8A8Error, match="1-D"):
        pkg.weights.shard_weight_scale("x.q_proj.weight", torch.ones(2, 2), 0, 1, None)


@pytest.mark.parametrize("world", [1, 2])
def test_moe_experts_are_stacked(pkg, oracle, world):
    """Per-expert gate/up/down tensors (HF layout) are sharded, merged into
    gate_up_proj, quantised per output channel of the unsharded weight and
    stacked over the experts under the MoELayer's state-dict names."""
    E, H, I = 4, 64, 32
    g = torch.Generator().manual_seed(5)
    p = "model.layers.0.mlp."
    items, full = [], {}
    for e in range(E):
        for proj, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            w = (torch.randn(*shape, generator=g) * 0.02).bfloat16()
            full[(e, proj)] = w
            items.append((f"{p}experts.{e}.{proj}.weight", w))
    items.append((p + "gate.weight", (torch.randn(E, H, generator=g) * 0.02).bfloat16()))
    for r in range(world):
        got = pkg.load_w8a8_state_dict(items, r, world, None, quantise=oracle.quant_weight_per_channel,
                                       num_experts=E)
        assert sorted(k for k in got if ".experts." in k) == [
            p + "experts.down_proj", p + "experts.down_proj_scale", p + "experts.gate_up_proj",
            p + "experts.gate_up_proj_scale"]
        il = I // world
        assert tuple(got[p + "experts.gate_up_proj"].shape) == (E, 2 * il, H)
        assert tuple(got[p + "experts.down_proj"].shape) == (E, H, il)
        assert tuple(got[p + "experts.down_proj_scale"].shape) == (E, H)
        for e in range(E):
            qg, sg = oracle.quant_weight_per_channel(full[(e, "gate_proj")])
            qu, su = oracle.quant_weight_per_channel(full[(e, "up_proj")])
            qd, sd = oracle.quant_weight_per_channel(full[(e, "down_proj")])
            sl = slice(r * il, (r + 1) * il)
            assert torch.equal(got[p + "experts.gate_up_proj"][e], torch.cat([qg[sl], qu[sl]]))
            assert torch.equal(got[p + "experts.gate_up_proj_scale"][e], torch.cat([sg[sl], su[sl]]))
            assert torch.equal(got[p + "experts.down_proj"][e], qd[:, sl])
            assert torch.equal(got[p + "experts.down_proj_scale"][e], sd)
        # the router (a LinearReplicated) is quantised whole on every rank
        qr, sr = oracle.quant_weight_per_channel(items[-1][1])
        assert torch.equal(got[p + "gate.weight"], qr) and torch.equal(got[p + "gate.weight_scale"], sr)
    with pytest.raises(pkg.W8A8Error):
        pkg.load_w8a8_state_dict(items[:-4], 0, 1, None, quantise=oracle.quant_weight_per_channel, num_experts=E)
