"""CPU, world_size 2 over gloo: the host-side tensor-parallel logic.

* the all-reduce plugin stack (DistributedCommunicator -> TorchDistributedImpl)
  on the known answers of the reference's tests/kernel/test_comm.py:96-149;
* the row-parallel composition (per-rank K-shard partials, then the plugin's
  all_reduce) against the oracle's tp_linear;
* the peer-memory communicator's handle exchange and open order, with a fake
  of the C ABI (the real one needs GPUs);
* failure detection on the host: a rank that never joins makes the other
  rank's collective fail with a timeout error instead of hanging.
"""
from __future__ import annotations

import ctypes
import multiprocessing as mp
import os
import sys
import traceback

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, scenario, q):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import importlib
        from datetime import timedelta

        import torch.distributed as dist

        timeout = timedelta(seconds=5 if scenario == "missing_rank" else 60)
        if scenario == "missing_rank" and rank == 1:
            q.put((rank, "ok", "skipped join"))
            return
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
        pkg = importlib.import_module("mini-sglang-fork_b200")
        from oracle import w8a8_oracle as O

        res = globals()["_scn_" + scenario](pkg, O, rank, world, dist)
        dist.destroy_process_group()
        q.put((rank, "ok", res))
    except BaseException:  # noqa: BLE001
        q.put((rank, "error", traceback.format_exc()))


def _run(scenario, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29300 + (os.getpid() + hash(scenario)) % 300
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, st, payload = q.get(timeout=timeout)
            out[r] = (st, payload)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    return out


def _ok(out):
    errs = {r: v[1] for r, v in out.items() if v[0] != "ok"}
    assert not errs, "\n".join(f"rank {r}:\n{e}" for r, e in errs.items())
    return {r: v[1] for r, v in out.items()}


# ------------------------------------------------------------------ scenarios
def _scn_plugin_known_answers(pkg, O, rank, world, dist):
    D = pkg.distributed
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]
    comm = D.DistributedCommunicator()
    n = 4096
    x = torch.ones(n, dtype=torch.bfloat16)
    for _ in range(4):
        x = comm.all_reduce(x)
    assert torch.all(x == world ** 4)
    x = comm.all_reduce(torch.full((n,), rank, dtype=torch.bfloat16))
    assert torch.all(x == world * (world - 1) // 2)
    x = comm.all_reduce(torch.cat([torch.zeros(n // 2), torch.ones(n // 2)]).bfloat16())
    assert torch.all(x[: n // 2] == 0) and torch.all(x[n // 2:] == world)
    # all_gather ordering (test_comm.py:141-149)
    g = comm.all_gather(torch.full((8,), rank, dtype=torch.bfloat16))
    assert torch.equal(g, torch.arange(world, dtype=torch.bfloat16).repeat_interleave(8))
    return True


def _scn_row_parallel_composition(pkg, O, rank, world, dist):
    """Each rank's W8A8 partial of its K-shard, summed by the plugin's
    all_reduce, equals the oracle's tensor-parallel row-parallel linear (on
    quantisation-exact inputs, where every sum is exact in any order)."""
    D = pkg.distributed
    D.reset_tp_info()
    D.set_tp_info(rank, world)
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]
    x, w = O.exact_quant_inputs(6, 64, 32, seed=5)
    wq, ws = O.quant_weight_per_channel(w)
    want = O.tp_linear("row", x, wq, ws, world)[rank]
    part = O.w8a8_linear(x.chunk(world, dim=1)[rank], O.shard_tensor(".down_proj", wq, rank, world, None), ws)[3]
    got = D.DistributedCommunicator().all_reduce(part.float()).bfloat16()
    assert torch.equal(got, want)
    # the layer classes size their shards from the same TP info
    layer = pkg.LinearRowParallel(64, 32, has_bias=False)
    assert (layer.local_input_size, layer.local_output_size) == (64 // world, 32)
    assert tuple(layer.weight.shape) == (32, 64 // world) and layer.weight.dtype == torch.int8
    assert tuple(layer.weight_scale.shape) == (32,)
    qkv = pkg.LinearQKVMerged(64, 8, 4, 1, has_bias=True)   # kv heads replicated (1 < tp)
    assert qkv.local_output_size == (4 // world + 2) * 8
    return True


def _tag(rank, world):
    return f"rank{rank:02d}/w{world:02d}".encode().ljust(16, b".")


class _FakeLib:
    """Stand-in for the C ABI's communicator entry points (records calls)."""

    def __init__(self, rank):
        self.rank = rank
        self.opened_with = None

    def w8a8_comm_handle_bytes(self):
        return 16

    def w8a8_comm_create(self, rank, world, dev, max_bytes, out_handle, blob):
        ctypes.memmove(blob, _tag(rank, world), 16)
        out_handle._obj.value = 1000 + rank
        return 0

    def w8a8_comm_open_peers(self, handle, buf):
        self.opened_with = bytes(buf.raw)
        return 0

    def w8a8_comm_set_timeout_ms(self, handle, ms):
        return 0

    def w8a8_comm_destroy(self, handle):
        pass

    def w8a8_last_error(self):
        return b""


def _scn_handle_exchange(pkg, O, rank, world, dist):
    fake = _FakeLib(rank)
    c = pkg.comm.PeerMemCommunicator(rank, world, 1 << 20, cpu_group=None, device=torch.device("cpu"),
                                     lib=fake, timeout_ms=500)
    blobs = [fake.opened_with[i * 16:(i + 1) * 16] for i in range(world)]
    assert blobs == [_tag(r, world) for r in range(world)]
    c.close()
    return True


def _scn_missing_rank(pkg, O, rank, world, dist):  # only rank 0 gets here
    raise AssertionError("init_process_group should have timed out")


# ---------------------------------------------------------------------- tests
def test_plugin_known_answers_gloo():
    _ok(_run("plugin_known_answers"))


def test_row_parallel_composition_gloo():
    _ok(_run("row_parallel_composition"))


def test_peer_mem_handle_exchange_order_gloo():
    _ok(_run("handle_exchange"))


def test_rank_that_never_joins_times_out():
    out = _run("missing_rank", timeout=120)
    assert out[1][0] == "ok"
    assert out[0][0] == "error"
    assert "timed out" in out[0][1].lower() or "timeout" in out[0][1].lower()


# ---------------------------------------------------------------- binding to the reference's own state
def _fresh_reference_modules(monkeypatch):
    """The reference's minisgl.distributed: the real package when
    MINISGL_PYTHON names mini-sglang's python/ directory (or it is already
    importable), else None."""
    import importlib
    import sys

    path = os.environ.get("MINISGL_PYTHON")
    if path:
        monkeypatch.syspath_prepend(path)
    try:
        ref = importlib.import_module("minisgl.distributed")
    except ImportError:
        return None
    info = sys.modules["minisgl.distributed.info"]
    monkeypatch.setattr(info, "_TP_INFO", None)
    monkeypatch.setattr(ref.DistributedCommunicator, "plugins", list(ref.DistributedCommunicator.plugins))
    return ref


def _stand_in_reference(monkeypatch):
    """A minimal module with the reference's distributed surface
    (set_tp_info / get_tp_info / try_get_tp_info / DistributedCommunicator
    with a class-level plugin list), registered as minisgl.distributed."""
    import sys
    import types

    mod = types.ModuleType("minisgl.distributed")
    state = {"info": None}

    class Info:
        def __init__(self, rank, size):
            self.rank, self.size = rank, size

    class Communicator:
        plugins = []

        def all_reduce(self, x):
            return self.plugins[-1].all_reduce(x)

    def set_tp_info(rank, size):
        state["info"] = Info(rank, size)

    mod.set_tp_info = set_tp_info
    mod.get_tp_info = lambda: state["info"]
    mod.try_get_tp_info = lambda: state["info"]
    mod.DistributedCommunicator = Communicator
    pkg = types.ModuleType("minisgl")
    pkg.__path__ = []
    monkeypatch.setitem(sys.modules, "minisgl", pkg)
    monkeypatch.setitem(sys.modules, "minisgl.distributed", mod)
    return mod


def _check_layers_follow_reference(pkg, ref, monkeypatch):
    D = pkg.distributed
    D.reset_tp_info()
    ref.set_tp_info(1, 4)  # the reference engine's call (M/engine/engine.py:32); none to this package
    assert D.get_tp_info().size == 4 and D.get_tp_info().rank == 1
    qkv = pkg.LinearQKVMerged(5120, 128, 64, 8, has_bias=False)
    gate_up = pkg.LinearColParallelMerged(5120, [25600, 25600], has_bias=False)
    down = pkg.LinearRowParallel(25600, 5120, has_bias=False)
    assert tuple(qkv.weight.shape) == ((16 + 2 * 2) * 128, 5120)
    assert tuple(gate_up.weight.shape) == (12800, 5120)
    assert tuple(down.weight.shape) == (5120, 6400) and tuple(down.weight_scale.shape) == (5120,)
    # the row-parallel fallback reduce goes through the reference's dispatcher
    assert isinstance(down._comm, ref.DistributedCommunicator)
    seen = []

    class Probe:
        def all_reduce(self, x):
            seen.append(x)
            return x

    ref.DistributedCommunicator.plugins.append(Probe())
    t = torch.ones(3)
    assert down._comm.all_reduce(t) is t and seen == [t]
    # enable_peer_mem_distributed registers its plugin with the reference's list too
    created = []

    class FakeComm:
        def __init__(self, rank, world, max_bytes, group, device=None, device_group=None):
            created.append((rank, world))

        def close(self):
            pass

    monkeypatch.setattr(pkg.comm, "PeerMemCommunicator", FakeComm)
    D.enable_peer_mem_distributed(D.get_tp_info(), None, max_bytes=1024)
    assert created == [(1, 4)]
    assert isinstance(ref.DistributedCommunicator.plugins[-1], D.PeerMemDistributedImpl)
    D.destroy_distributed()
    assert not any(isinstance(p, D.PeerMemDistributedImpl) for p in ref.DistributedCommunicator.plugins)
    D.DistributedCommunicator.plugins = [D.TorchDistributedImpl()]


def test_layers_follow_a_reference_style_distributed_module(pkg, monkeypatch):
    ref = _stand_in_reference(monkeypatch)
    _check_layers_follow_reference(pkg, ref, monkeypatch)
    # this package's own set_tp_info takes precedence once called
    pkg.distributed.set_tp_info(0, 2)
    assert pkg.distributed.get_tp_info().size == 2
    pkg.distributed.reset_tp_info()


def test_layers_follow_the_reference_distributed_state(pkg, monkeypatch):
    ref = _fresh_reference_modules(monkeypatch)
    if ref is None:
        pytest.skip("mini-sglang is not importable here (set MINISGL_PYTHON to its python/ directory)")
    _check_layers_follow_reference(pkg, ref, monkeypatch)
