"""GPU: quantise-at-load with the library's CUDA quantiser (the loader's
default) gives exactly the oracle's shards, and a layer loaded from the
stream computes the oracle's forward bit for bit."""
from __future__ import annotations

import pytest
import torch

from test_weights_cpu import HD, HIDDEN, NKV, NQ, _checkpoint, _expected

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [1, 4])
def test_cuda_quantise_at_load_matches_oracle(pkg, oracle, cuda_dev, world):
    items = _checkpoint(seed=11, layers=1)
    for r in range(world):
        got = pkg.load_w8a8_state_dict(items, r, world, NKV, device=cuda_dev)
        want = _expected(oracle, items, r, world)
        assert sorted(got) == sorted(want)
        for k, v in want.items():
            assert got[k].dtype == v.dtype, k
            assert torch.equal(got[k].cpu(), v), k
        assert got["model.layers.0.mlp.gate_up_proj.weight"].is_cuda


def test_loaded_layer_forward_matches_oracle(pkg, oracle, cuda_dev):
    D = pkg.distributed
    items = _checkpoint(seed=13, layers=1)
    D.reset_tp_info()
    D.set_tp_info(0, 1)
    try:
        sd = pkg.load_w8a8_state_dict(items, 0, 1, NKV, device=cuda_dev)
        layer = pkg.LinearQKVMerged(HIDDEN, HD, NQ, NKV, has_bias=True)
        prefix = "model.layers.0.self_attn.qkv_proj"
        layer.load_state_dict({k: v.to(cuda_dev) for k, v in sd.items() if k.startswith(prefix + ".")},
                              prefix=prefix)
        x = torch.randn(37, HIDDEN, generator=torch.Generator().manual_seed(1)).bfloat16()
        y = layer.forward(x.to(cuda_dev))
        want = oracle.w8a8_linear(x, sd[prefix + ".weight"].cpu(), sd[prefix + ".weight_scale"].cpu(),
                                  sd[prefix + ".bias"].cpu())[3]
        assert torch.equal(y.cpu(), want)
        assert y.shape == (37, (NQ + 2 * NKV) * HD)
    finally:
        D.reset_tp_info()
