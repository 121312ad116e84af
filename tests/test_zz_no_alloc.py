"""GPU: w8a8_gemm_static_scratch, the GEMM entry point that allocates nothing
(stream-K scratch in a fixed 20 MiB device array), called through the C ABI
and compared with w8a8_gemm given a caller workspace.  Two calls in a row per
shape: the second one reuses the counters the first left behind.

Collected last on purpose (file name), and must also pass alone in a fresh
process: the first call on the device does the scratch set-up.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

# (M, N, K, bias): stream-K plans with cut tiles on 16-, 64- and 128-wide
# tiles (2.7 / 10 / 19.7 MB of scratch on 148 SMs), a single token, and a
# whole-block plan that uses no scratch.
CASES = [(16, 5120, 25600, False), (48, 2048, 8192, True), (200, 5120, 1024, True),
         (1, 5120, 5120, False), (4096, 5120, 512, True)]


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _inputs(m, n, k, bias, dev):
    g = torch.Generator().manual_seed(m * 131 + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sa = torch.rand(m, generator=g) * 1e-3 + 1e-4
    sb = torch.rand(n, generator=g) * 1e-3 + 1e-4
    bb = (torch.randn(n, generator=g) * 0.1).bfloat16() if bias else None
    return [None if t is None else t.to(dev) for t in (a, b, sa, sb, bb)]


@pytest.mark.parametrize("m,n,k,bias", CASES)
def test_static_scratch_matches_workspace_entry_point(pkg, cuda_dev, m, n, k, bias):
    lib = pkg.load_library()
    L = pkg._lib
    a, b, sa, sb, bb = _inputs(m, n, k, bias, cuda_dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)

    ref = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_dev)
    ref_i32 = torch.empty(m, n, dtype=torch.int32, device=cuda_dev)
    ws = pkg.ops.gemm_workspace(cuda_dev)
    st = lib.w8a8_gemm(_p(a), _p(b), _p(sa), _p(sb), _p(bb), _p(ref), _p(ref_i32), m, n, k,
                       _p(ws), ws.numel(), stream)
    assert st == L.OK, lib.w8a8_last_error()

    for call in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
        out_i32 = torch.full((m, n), -1, dtype=torch.int32, device=cuda_dev)
        st = lib.w8a8_gemm_static_scratch(_p(a), _p(b), _p(sa), _p(sb), _p(bb), _p(out), _p(out_i32),
                                          m, n, k, stream)
        assert st == L.OK, lib.w8a8_last_error()
        torch.cuda.synchronize(cuda_dev)
        assert torch.equal(out_i32, ref_i32), f"call {call}: int32 accumulators differ"
        torch.testing.assert_close(out, ref, atol=0, rtol=0, msg=f"call {call}: bf16 output differs")
    assert pkg.ops.device_error() == 0


def test_static_scratch_rejects_plans_above_its_size(pkg, cuda_dev):
    """A plan needing more stream-K scratch than the static 20 MiB is refused on
    the host, before any launch.  On a 148-SM B200 no plan of the planner needs
    that much (largest: 19.7 MB, 128 x 128 tiles with a cut remainder); a
    device with more SMs can produce one."""
    lib = pkg.load_library()
    L = pkg._lib
    limit = 20 * 2 ** 20
    shapes = [(m, n, k) for m in (1, 17, 48, 65, 100, 128, 200, 256, 1024) for n in (1280, 5120, 51200)
              for k in (1024, 5120, 25600)]
    over = [(m, n, k) for (m, n, k) in shapes if pkg.ops.gemm_plan(m, n, k)["workspace_bytes"] > limit]
    if not over:
        pytest.skip("no plan on this device needs more than the static scratch")
    m, n, k = over[0]
    plan = pkg.ops.gemm_plan(m, n, k)
    a, b, sa, sb, _ = _inputs(8, 16, 16, False, cuda_dev)  # never read: the call stops on the host
    out = torch.empty(8, 16, dtype=torch.bfloat16, device=cuda_dev)
    st = lib.w8a8_gemm_static_scratch(_p(a), _p(b), _p(sa), _p(sb), None, _p(out), None, m, n, k,
                                      ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream))
    assert st == L.ERR_WORKSPACE
    msg = lib.w8a8_last_error()
    assert b"static maximum" in msg and str(plan["workspace_bytes"]).encode() in msg


def test_static_scratch_empty_batch(pkg, cuda_dev):
    """An empty batch is accepted without work, as in w8a8_gemm."""
    lib = pkg.load_library()
    assert lib.w8a8_gemm_static_scratch(None, None, None, None, None, None, None, 0, 5120, 1024, None) == pkg._lib.OK
