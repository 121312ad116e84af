"""GPU: the W8A8 layer classes (mini-sglang's operator surface) vs the oracle.

Every class is built through its reference constructor signature, loaded
through ``load_state_dict`` and run through ``forward``, at TP=1 on one GPU
(row-parallel TP>1 is covered in test_comm_gpu.py).  Also: the GatedMLP
composition with the fused SiLU*mul quantiser, CUDA-graph capture of a layer,
and the state-dict contract (keys, shape/dtype checks).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _tp1(pkg):
    pkg.reset_tp_info()
    pkg.set_tp_info(0, 1)
    pkg.DistributedCommunicator.plugins = [pkg.distributed.TorchDistributedImpl()]
    yield
    pkg.reset_tp_info()


def _weights(oracle, n, k, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    wq, ws = oracle.quant_weight_per_channel(w)
    b = (torch.randn(n, generator=g) * 0.1).bfloat16() if bias else None
    return wq, ws, b


def _load(layer, wq, ws, b, dev):
    sd = {"weight": wq.to(dev), "weight_scale": ws.to(dev)}
    if b is not None:
        sd["bias"] = b.to(dev)
    layer.load_state_dict(sd)


@pytest.mark.parametrize("m", [1, 7, 64, 300])
def test_each_layer_class_matches_oracle(pkg, oracle, cuda_dev, m):
    h, hd, nq, nkv, inter = 512, 64, 8, 2, 768
    layers = {
        "qkv": (pkg.LinearQKVMerged(h, hd, nq, nkv, has_bias=True), (nq + 2 * nkv) * hd, h, True),
        "o_proj": (pkg.LinearOProj(nq * hd, h, has_bias=False), h, nq * hd, False),
        "gate_up": (pkg.LinearColParallelMerged(h, [inter, inter], has_bias=False), 2 * inter, h, False),
        "down": (pkg.LinearRowParallel(inter, h, has_bias=False), h, inter, False),
        "replicated": (pkg.LinearReplicated(h, 256, has_bias=True), 256, h, True),
    }
    for i, (name, (layer, n, k, bias)) in enumerate(layers.items()):
        assert (layer.local_output_size, layer.local_input_size) == (n, k)
        wq, ws, b = _weights(oracle, n, k, seed=i + 10 * m, bias=bias)
        _load(layer, wq, ws, b, cuda_dev)
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + i)).bfloat16()
        y = layer.forward(x.to(cuda_dev))
        want = oracle.w8a8_linear(x, wq, ws, b)[3]
        assert y.dtype == torch.bfloat16 and tuple(y.shape) == (m, n)
        assert torch.equal(y.cpu(), want), name


def test_state_dict_contract(pkg, cuda_dev):
    layer = pkg.LinearColParallelMerged(64, [32, 32], has_bias=True)
    assert sorted(layer.state_dict().keys()) == ["bias", "weight", "weight_scale"]
    with pytest.raises(ValueError):
        layer.load_state_dict({"weight": torch.zeros(64, 64, dtype=torch.bfloat16),
                               "weight_scale": torch.zeros(64), "bias": torch.zeros(64, dtype=torch.bfloat16)})
    with pytest.raises(RuntimeError, match="Unexpected keys"):
        layer.load_state_dict({"weight": torch.zeros(64, 64, dtype=torch.int8),
                               "weight_scale": torch.zeros(64), "bias": torch.zeros(64, dtype=torch.bfloat16),
                               "extra": torch.zeros(1)})


def test_gated_mlp_matches_oracle(pkg, oracle, cuda_dev):
    h, inter, m = 512, 1024, 33
    mlp = pkg.GatedMLP(h, inter)
    wgu, sgu, _ = _weights(oracle, 2 * inter, h, seed=1)
    wd, sd, _ = _weights(oracle, h, inter, seed=2)
    _load(mlp.gate_up_proj, wgu, sgu, None, cuda_dev)
    _load(mlp.down_proj, wd, sd, None, cuda_dev)
    assert sorted(mlp.state_dict().keys()) == ["down_proj.weight", "down_proj.weight_scale",
                                               "gate_up_proj.weight", "gate_up_proj.weight_scale"]
    x = torch.randn(m, h, generator=torch.Generator().manual_seed(3)).bfloat16()
    y = mlp.forward(x.to(cuda_dev))
    gu = oracle.w8a8_linear(x, wgu, sgu)[3]
    # the fused kernel's own bf16 SiLU*mul product (expf may differ by an ulp
    # from the CPU's) is what its quantiser saw: check quant + down on it
    qa, prod = pkg.ops.silu_and_mul_quant(gu.to(cuda_dev), with_bf16=True)
    q_ref, s_ref = oracle.quant_per_token(prod.cpu())
    want = oracle.dequant(oracle.int_gemm(q_ref, wd), s_ref, sd)
    assert torch.equal(y.cpu(), want)
    # and the end result stays within the north-star tolerance of the pure-CPU chain
    full = oracle.w8a8_linear(oracle.silu_and_mul(gu), wd, sd)[3]
    torch.testing.assert_close(y.cpu().float(), full.float(), rtol=1e-2, atol=1e-2)


def test_layer_forward_under_cuda_graph(pkg, oracle, cuda_dev):
    """The path is capturable: quantiser + GEMM replayed from a CUDA graph give
    the oracle's result for fresh inputs every replay."""
    h, n, m = 1024, 2048, 16
    layer = pkg.LinearColParallelMerged(h, [n // 2, n // 2], has_bias=False)
    wq, ws, _ = _weights(oracle, n, h, seed=5)
    _load(layer, wq, ws, None, cuda_dev)
    x = torch.zeros(m, h, dtype=torch.bfloat16, device=cuda_dev)
    stream = torch.cuda.Stream(cuda_dev)
    with torch.cuda.stream(stream):
        layer.forward(x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        y = layer.forward(x)
    for i in range(3):
        xi = torch.randn(m, h, generator=torch.Generator().manual_seed(100 + i)).bfloat16()
        x.copy_(xi)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y.cpu(), oracle.w8a8_linear(xi, wq, ws)[3]), i
    del g
    assert pkg.ops.device_error() == 0


def test_quantized_activation_input(pkg, oracle, cuda_dev):
    """A QuantizedActivation (from the fused SiLU*mul quantiser) is accepted by
    every layer's forward in place of bf16."""
    layer = pkg.LinearRowParallel(256, 128, has_bias=False)
    wq, ws, _ = _weights(oracle, 128, 256, seed=8)
    _load(layer, wq, ws, None, cuda_dev)
    x = torch.randn(9, 256, generator=torch.Generator().manual_seed(9)).bfloat16()
    q, s = pkg.ops.quant_per_token(x.to(cuda_dev))
    y = layer.forward(pkg.QuantizedActivation(q, s))
    assert torch.equal(y.cpu(), oracle.w8a8_linear(x, wq, ws)[3])
