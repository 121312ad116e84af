"""GPU, 2+ devices: the NVLink peer-memory all-reduce and the fused row-parallel
GEMM + all-reduce, one process per GPU (spawned), CPU group over gloo.

Known answers follow the reference's tests/kernel/test_comm.py:96-135 (ones
reduced 4 times -> world**4; full(rank) -> world*(world-1)/2 with rank 0
lagging 1 s; half zeros / half ones).  Random data and the fused GEMM are
compared bit for bit with the CPU oracle (fp32 rank-order sum of the ranks'
bf16 partials, one rounding).  The failure path makes one rank skip a
collective so the other's bounded flag wait runs out (short limit) and the
status is read back on the host — no GPU fault, no hang.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import sys
import traceback

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _world():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return min(n, 8)


def _worker(rank, world, port, scenario, q):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import importlib
        from datetime import timedelta

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        pkg = importlib.import_module("mini-sglang-fork_b200")
        from oracle import w8a8_oracle as O

        result = globals()["_scn_" + scenario](pkg, O, rank, world, dev, dist)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", result))
    except BaseException:  # noqa: BLE001 - reported to the parent
        q.put((rank, "error", traceback.format_exc()))


def _run(scenario, world=None, timeout=240):
    world = world or _world()
    if world < 2:
        pytest.skip("needs >= 2 CUDA devices")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() % 200)
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=timeout)
            results[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    errors = {r: v[1] for r, v in results.items() if v[0] != "ok"}
    assert not errors, "\n".join(f"rank {r}:\n{e}" for r, e in errors.items())
    return {r: v[1] for r, v in results.items()}


# ------------------------------------------------------------------ scenarios
def _scn_known_answers(pkg, O, rank, world, dev, dist):
    import time

    comm = pkg.comm.PeerMemCommunicator(rank, world, 8192 * 512 * 2, device=dev)
    for mode, numel in ((0, 8192 * 512), (0, 4096), (1, 8192 * 512), (2, 8192 * 512), (2, 4096 + 8)):
        comm.set_mode(mode)  # automatic, forced one-shot, forced two-shot
        x = torch.ones(numel, dtype=torch.bfloat16, device=dev)
        for _ in range(4):
            comm.all_reduce(x)
        assert torch.all(x == world ** 4), "ones^4"
        x = torch.full((numel,), rank, dtype=torch.bfloat16, device=dev)
        if rank == 0:
            torch.cuda.synchronize()
            time.sleep(1)  # the others must wait (bounded) for the lagging rank
        comm.all_reduce(x)
        assert torch.all(x == world * (world - 1) // 2), "rank sum"
        x = torch.cat([torch.zeros(numel // 2, dtype=torch.bfloat16, device=dev),
                       torch.ones(numel // 2, dtype=torch.bfloat16, device=dev)])
        comm.all_reduce(x)
        assert torch.all(x[: numel // 2] == 0) and torch.all(x[numel // 2:] == world), "half ones"
    assert comm.device_error() == 0
    comm.close()
    return True


def _scn_random_bit_exact(pkg, O, rank, world, dev, dist):
    comm = pkg.comm.PeerMemCommunicator(rank, world, 1 << 24, device=dev)
    for mode in (1, 2):
        comm.set_mode(mode)
        for numel in (8, 1000 * 8, 5120 * 7, 4096 * 1024):
            parts = [torch.randn(numel, generator=torch.Generator().manual_seed(numel + r)).bfloat16()
                     for r in range(world)]
            want = O.all_reduce_sum(parts)
            x = parts[rank].to(dev)
            comm.all_reduce(x)
            assert torch.equal(x.cpu(), want), f"mode={mode} numel={numel}"
    assert comm.device_error() == 0
    comm.close()
    return True


def _scn_gemm_allreduce(pkg, O, rank, world, dev, dist):
    """Fused row-parallel GEMM + all-reduce == oracle tp_linear("row"), bit-exact."""
    comm = pkg.comm.PeerMemCommunicator(rank, world, 2560 * 5120 * 2, device=dev)
    cases = [(0, 1, 5120, 1024 * world, False), (0, 16, 4096, 512 * world, True),
             (0, 64, 1024, 256 * world, False), (0, 200, 2048, 384 * world, False),
             (0, 1024, 5120, 512 * world, False), (0, 2048, 1536, 128 * world, True),
             # forced one-shot and two-shot reductions on normal-orientation tiles
             (1, 333, 4096, 256 * world, False), (2, 333, 4096, 256 * world, True),
             (2, 1024, 5120, 512 * world, False), (2, 65, 2048, 128 * world, False),
             # large M selects the 2-SM pair kernel (256x256 per CTA pair)
             (0, 2560, 5120, 128 * world, True), (1, 2500, 5120, 128 * world, False),
             (2, 2560, 5120, 128 * world, False)]
    for (mode, m, n, kfull, bias) in cases:
        comm.set_mode(mode)
        g = torch.Generator().manual_seed(m * 7 + n)
        x = torch.randn(m, kfull, generator=g).bfloat16()
        w = (torch.randn(n, kfull, generator=g) * 0.02).bfloat16()
        b = (torch.randn(n, generator=g) * 0.1).bfloat16() if bias else None
        wq, ws = O.quant_weight_per_channel(w)
        want = O.tp_linear("row", x, wq, ws, world, bias=b)[rank]
        xs = x.chunk(world, dim=1)[rank].contiguous().to(dev)
        wshard = O.shard_tensor(".down_proj", wq, rank, world, None).to(dev)
        q, s = pkg.ops.quant_per_token(xs)
        y = comm.gemm_allreduce(q, wshard, s, ws.to(dev), None if b is None else b.to(dev))
        torch.cuda.synchronize()
        assert torch.equal(y.cpu(), want), f"mode={mode} m={m} n={n} k={kfull}"
    assert comm.device_error() == 0
    comm.close()
    return True


def _scn_gemm_allreduce_cfg3(pkg, O, rank, world, dev, dist):
    """The benchmarked row-parallel shapes at M = 4096 (cfg3 o_proj K=8192 and
    down K=25600, sharded over the world): the fused GEMM + all-reduce output
    on two sampled rows of every 128-row tile is bit-exact with the oracle's
    tp_linear("row"), and identical on every rank."""
    m, n = 4096, 5120
    rows = []
    for t in range(m // 128):
        rows += [t * 128 + (t * 53 + 17) % 128, t * 128 + 127]
    idx = torch.tensor(rows, device=dev)
    comm = pkg.comm.PeerMemCommunicator(rank, world, m * n * 2, device=dev)
    digests = []
    for kfull in (8192, 25600):
        g = torch.Generator(device=dev).manual_seed(kfull)  # the same full tensors on every rank
        x = torch.randn(m, kfull, device=dev, generator=g).bfloat16()
        wq, ws = pkg.ops.quant_per_token((torch.randn(n, kfull, device=dev, generator=g) * 0.02).bfloat16())
        kl = kfull // world
        xs = x[:, rank * kl:(rank + 1) * kl].contiguous()
        wshard = wq[:, rank * kl:(rank + 1) * kl].contiguous()
        q, s = pkg.ops.quant_per_token(xs)
        y = comm.gemm_allreduce(q, wshard, s, ws)
        torch.cuda.synchronize()
        want = O.tp_linear("row", x.index_select(0, idx).cpu(), wq.cpu(), ws.cpu(), world)[rank]
        got = y.index_select(0, idx).cpu()
        assert torch.equal(got, want), f"k={kfull}: max |diff| {float((got.float() - want.float()).abs().max())}"
        digests.append(float(y.float().sum()))
    everyone = [None] * world
    dist.all_gather_object(everyone, digests)
    assert all(d == digests for d in everyone), "ranks disagree on the reduced output"
    assert comm.device_error() == 0
    comm.close()
    return True


def _scn_gemm_allreduce_nvls(pkg, O, rank, world, dev, dist):
    """The fused GEMM + all-reduce with the two-shot reduce through the
    NVSwitch (mode 3: partials stay local, each row share is summed in the
    switch by multimem.ld_reduce with fp32 accumulation and multicast back).
    The switch adds in its own order and rounds its fp32 sum to bf16 by its
    own rule (exact ties of a two-rank sum do not always round to even), so
    the bf16 result is checked within one bf16 ulp of the oracle (and the 1e-2
    contract bound) and identical on every rank; the fraction of elements that
    differ from the rank-order sum is returned."""
    comm = pkg.comm.PeerMemCommunicator(rank, world, 4096 * 5120 * 2, device=dev)
    assert comm.nvls, f"no multicast buffer: {comm.nvls_error}"
    comm.set_mode(3)
    cases = [(333, 4096, 256 * world, True), (1024, 5120, 512 * world, False), (2560, 5120, 128 * world, False),
             (4096, 5120, 8192, False), (65, 2048, 128 * world, True)]
    digests, fractions = [], []
    for (m, n, kfull, bias) in cases:
        g = torch.Generator().manual_seed(m * 11 + n)
        x = torch.randn(m, kfull, generator=g).bfloat16()
        w = (torch.randn(n, kfull, generator=g) * 0.02).bfloat16()
        b = (torch.randn(n, generator=g) * 0.1).bfloat16() if bias else None
        wq, ws = O.quant_weight_per_channel(w)
        want = O.tp_linear("row", x, wq, ws, world, bias=b)[rank].float()
        xs = x.chunk(world, dim=1)[rank].contiguous().to(dev)
        wshard = O.shard_tensor(".down_proj", wq, rank, world, None).to(dev)
        q, s = pkg.ops.quant_per_token(xs)
        for rep in range(2):  # both halves of the buffer
            y = comm.gemm_allreduce(q, wshard, s, ws.to(dev), None if b is None else b.to(dev))
            torch.cuda.synchronize()
            got = y.cpu().float()
            diff = (got - want).abs()
            assert torch.all(diff <= want.abs() * 2.0 ** -7 + 1e-30), (m, n, kfull, float(diff.max()))
            torch.testing.assert_close(got, want, rtol=1e-2, atol=1e-2)
            fractions.append(round(float((diff != 0).float().mean()), 5))
        digests.append(float(y.float().sum()))
    everyone = [None] * world
    dist.all_gather_object(everyone, digests)
    assert all(d == digests for d in everyone), "ranks disagree on the reduced output"
    assert comm.device_error() == 0
    comm.close()
    return fractions


def _scn_broadcast(pkg, O, rank, world, dev, dist):
    """Peer-memory broadcast from every root, at sizes from one vector to
    42 MB (the bench's e2e input), twice per size (both buffer halves)."""
    comm = pkg.comm.PeerMemCommunicator(rank, world, 4096 * 5120 * 2, device=dev)
    for root in range(world):
        for numel in (8, 4096 + 8, 4096 * 5120):
            for rep in range(2):
                want = torch.randn(numel, generator=torch.Generator().manual_seed(numel + root + rep)).bfloat16()
                x = want.to(dev) if rank == root else torch.full((numel,), -3.0, dtype=torch.bfloat16, device=dev)
                comm.broadcast(x, root=root)
                assert torch.equal(x.cpu(), want), f"root={root} numel={numel} rep={rep}"
    assert comm.device_error() == 0
    comm.close()
    return True


def _scn_layers_and_graphs(pkg, O, rank, world, dev, dist):
    """LinearRowParallel / LinearOProj through enable_peer_mem_distributed, eager
    and replayed from a CUDA graph (device-side epochs keep replays correct)."""
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(rank, world)
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]
    comm = D.enable_peer_mem_distributed(D.get_tp_info(), None, max_bytes=64 * 5120 * 2, device=dev)
    h, inter, m = 1024, 512 * world, 48
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(h, inter, generator=g) * 0.02).bfloat16()
    wq, ws = O.quant_weight_per_channel(w)
    layer = pkg.LinearRowParallel(inter, h, has_bias=False)
    layer.load_state_dict({"weight": O.shard_tensor(".down_proj", wq, rank, world, None).to(dev),
                           "weight_scale": ws.to(dev)})
    xs = [torch.randn(m, inter, generator=torch.Generator().manual_seed(10 + i)).bfloat16() for i in range(3)]
    x_dev = torch.empty(m, inter // world, dtype=torch.bfloat16, device=dev)
    x_dev.copy_(xs[0].chunk(world, dim=1)[rank])
    y = layer.forward(x_dev)
    assert torch.equal(y.cpu(), O.tp_linear("row", xs[0], wq, ws, world)[rank]), "eager"
    # plugin all_reduce also goes through the peer-memory communicator
    z = torch.full((4096,), rank + 1, dtype=torch.bfloat16, device=dev)
    D.DistributedCommunicator().all_reduce(z)
    assert torch.all(z == world * (world + 1) // 2)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        layer.forward(x_dev)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        y_g = layer.forward(x_dev)
    for i in range(3):
        x_dev.copy_(xs[i].chunk(world, dim=1)[rank])
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y_g.cpu(), O.tp_linear("row", xs[i], wq, ws, world)[rank]), f"replay {i}"
    del graph
    assert comm.device_error() == 0
    D.destroy_distributed()
    return True


def _scn_vocab_embedding_allreduce(pkg, O, rank, world, dev, dist):
    """The embedding all-reduce of a vocabulary-parallel embedding (the
    reference's VocabParallelEmbedding, M/layers/embedding.py:20-42: each rank
    looks up its ceil(V/p) vocabulary rows, zero rows for ids outside them,
    then DistributedCommunicator.all_reduce) reaches the peer-memory all-reduce
    once the plugin is enabled.  One rank contributes each row, so the sum is
    the unsharded lookup exactly."""
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(rank, world)
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]
    comm = D.enable_peer_mem_distributed(D.get_tp_info(), None, max_bytes=1 << 21, device=dev)
    V, H, T = 1003, 5120, 97
    g = torch.Generator().manual_seed(11)
    table = torch.randn(V, H, generator=g).bfloat16()
    ids = torch.randint(0, V, (T,), generator=g)
    per = -(-V // world)
    start, end = per * rank, min(per * (rank + 1), V)
    local = table[start:end].to(dev)
    idd = ids.to(dev)
    inside = (idd >= start) & (idd < end)
    y = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
    y[inside] = local[idd[inside] - start]
    y = D.DistributedCommunicator().all_reduce(y)
    assert torch.equal(y.cpu(), table[ids])
    assert comm.device_error() == 0
    D.destroy_distributed()
    return True


def _scn_timeout_status(pkg, O, rank, world, dev, dist):
    """Rank 0 calls all_reduce while the other ranks do not: its bounded flag
    wait runs out after ~0.3 s and the host reads the error status."""
    comm = pkg.comm.PeerMemCommunicator(rank, world, 1 << 20, device=dev, timeout_ms=300)
    x = torch.ones(4096, dtype=torch.bfloat16, device=dev)
    comm.all_reduce(x)  # a normal call first
    torch.cuda.synchronize()
    dist.barrier()
    err = 0
    if rank == 0:
        comm.all_reduce(x)
        torch.cuda.synchronize()
        err = comm.device_error()
        assert err != 0, "timed-out wait must be reported"
        pkg.ops.device_error(clear=True)
        # the context is still usable
        assert float(torch.ones(8, device=dev).sum()) == 8.0
    dist.barrier()
    comm.close()
    return err


def _scn_fused_timeout_status(pkg, O, rank, world, dev, dist):
    """Rank 0 issues fused GEMM + all-reduce calls that the other ranks skip:
    its reduce groups' bounded flag waits run out (~0.3 s each) and the host
    reads the error status; the GEMM warps never wait on a flag, so the kernel
    ends by itself.  Both the pair kernel (M=2048) and a swap-AB tile (M=64)."""
    comm = pkg.comm.PeerMemCommunicator(rank, world, 2048 * 5120 * 2, device=dev, timeout_ms=300)
    g = torch.Generator().manual_seed(5)
    shapes = [(64, 1024, 256), (2048, 5120, 256)]
    ops = []
    for m, n, k in shapes:
        a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8).to(dev)
        w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).to(dev)
        sa, sw = (torch.rand(m, generator=g) * 1e-3).to(dev), (torch.rand(n, generator=g) * 1e-3).to(dev)
        ops.append((a, w, sa, sw))
    for a, w, sa, sw in ops:  # normal calls first, on every rank
        comm.gemm_allreduce(a, w, sa, sw)
    torch.cuda.synchronize()
    assert comm.device_error() == 0
    dist.barrier()
    errs = []
    if rank == 0:
        for a, w, sa, sw in ops:
            comm.gemm_allreduce(a, w, sa, sw)
            torch.cuda.synchronize()
            errs.append(comm.device_error())
            pkg.ops.device_error(clear=True)
        assert all(e != 0 for e in errs), errs
        assert float(torch.ones(8, device=dev).sum()) == 8.0  # the context is still usable
    dist.barrier()
    comm.close()
    return errs


# ---------------------------------------------------------------------- tests
def test_allreduce_known_answers():
    _run("known_answers")


def test_allreduce_random_bit_exact():
    _run("random_bit_exact")


def test_gemm_allreduce_bit_exact():
    _run("gemm_allreduce")


def test_gemm_allreduce_cfg3_shapes():
    _run("gemm_allreduce_cfg3", timeout=600)


def test_broadcast():
    _run("broadcast")


def test_gemm_allreduce_nvls():
    res = _run("gemm_allreduce_nvls", timeout=600)
    print("NVLS elements differing from the rank-order sum (fraction per case):", res[0])


def test_row_parallel_layer_and_cuda_graph():
    _run("layers_and_graphs")


def test_vocab_embedding_allreduce():
    _run("vocab_embedding_allreduce")


def test_flag_wait_timeout_reported():
    res = _run("timeout_status")
    assert res[0] != 0


def test_fused_flag_wait_timeout_reported():
    res = _run("fused_timeout_status")
    assert len(res[0]) == 2 and all(e != 0 for e in res[0])
