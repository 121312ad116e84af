"""CPU: the C-ABI library loads, exports every symbol include/w8a8_tp.h
declares, validates arguments on the host, and plans tiles — no GPU calls."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "w8a8_tp.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(w8a8_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    names = _declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    # the ctypes binding covers exactly the declared surface
    assert sorted(pkg._lib.SIGNATURES) == names


def test_abi_version_and_error_channel(pkg):
    lib = pkg.load_library()
    assert lib.w8a8_abi_version() == 1
    assert isinstance(lib.w8a8_last_error(), bytes)


def test_host_validation_rejects_bad_arguments(pkg):
    """Argument checks run on the host before any CUDA call."""
    lib = pkg.load_library()
    L = pkg._lib
    # null pointers / misaligned K are rejected with a status and a message
    st = lib.w8a8_quant_per_token(None, 16, None, None, 4, 16, None)
    assert st == L.ERR_INVALID_ARG and b"null" in lib.w8a8_last_error()
    st = lib.w8a8_quant_per_token(16, 12, 16, 16, 4, 12, None)
    assert st == L.ERR_INVALID_ARG and b"multiple of 8" in lib.w8a8_last_error()
    st = lib.w8a8_quant_per_token(24, 16, 16, 16, 4, 16, None)
    assert st == L.ERR_ALIGNMENT
    st = lib.w8a8_gemm(16, 16, 16, 16, None, 16, None, 8, 24, 40, None, 0, None)
    assert st == L.ERR_INVALID_ARG and b"multiple of 16" in lib.w8a8_last_error()
    st = lib.w8a8_gemm(16, 16, 16, 16, None, 16, None, 8, 20, 32, None, 0, None)
    assert st == L.ERR_INVALID_ARG
    st = lib.w8a8_gemm(16, 18, 16, 16, None, 16, None, 8, 32, 32, None, 0, None)
    assert st == L.ERR_ALIGNMENT
    st = lib.w8a8_silu_mul_quant(16, 10, 16, 16, None, 2, 12, None)
    assert st == L.ERR_INVALID_ARG
    # fused RMSNorm + quant: null weight, K % 8, K above 8192, residual_out without a residual
    st = lib.w8a8_rmsnorm_quant(16, 16, None, 16, None, 1e-6, 16, 16, None, None, 4, 16, None)
    assert st == L.ERR_INVALID_ARG and b"null" in lib.w8a8_last_error()
    st = lib.w8a8_rmsnorm_quant(16, 16, None, 16, 16, 1e-6, 16, 16, None, None, 4, 12, None)
    assert st == L.ERR_INVALID_ARG and b"multiple of 8" in lib.w8a8_last_error()
    st = lib.w8a8_rmsnorm_quant(16, 16384, None, 16, 16, 1e-6, 16, 16, None, None, 4, 16384, None)
    assert st == L.ERR_UNSUPPORTED and b"8192" in lib.w8a8_last_error()
    st = lib.w8a8_rmsnorm_quant(16, 16, None, 16, 16, 1e-6, 16, 16, 16, None, 4, 16, None)
    assert st == L.ERR_INVALID_ARG and b"residual_out" in lib.w8a8_last_error()
    st = lib.w8a8_rmsnorm_quant(16, 16, 16, 16, 16, 1e-6, 16, 16, None, None, 4, 16, None)
    assert st == L.ERR_INVALID_ARG and b"residual_out" in lib.w8a8_last_error()
    st = lib.w8a8_rmsnorm_quant(16, 16, None, 16, 16, -1.0, 16, 16, None, None, 4, 16, None)
    assert st == L.ERR_INVALID_ARG and b"eps" in lib.w8a8_last_error()
    assert lib.w8a8_rmsnorm_quant(None, 16, None, 16, None, 1e-6, None, None, None, None, 0, 16, None) == L.OK
    # empty batches are a no-op success, as F.linear on an empty input
    assert lib.w8a8_quant_per_token(None, 16, None, None, 0, 16, None) == L.OK
    assert lib.w8a8_silu_mul_quant(None, 32, None, None, None, 0, 16, None) == L.OK
    assert lib.w8a8_gemm_config(16, 16, 16, 16, None, 16, None, 0, 32, 32, 0, 0, None, 0, None) == L.OK
    assert lib.w8a8_gemm_config(16, 16, 16, 16, None, 16, None, 8, 32, 32, 8, 0, None, 0, None) == L.ERR_INVALID_ARG
    # silu_mul_quant: q and scale come together; the bf16-only form needs y_out
    st = lib.w8a8_silu_mul_quant(16, 32, 16, None, 16, 2, 16, None)
    assert st == L.ERR_INVALID_ARG and b"together" in lib.w8a8_last_error()
    st = lib.w8a8_silu_mul_quant(16, 32, None, None, None, 2, 16, None)
    assert st == L.ERR_INVALID_ARG and b"nothing to write" in lib.w8a8_last_error()
    # gate_up GEMM with the SiLU epilogue and the quantiser with a known absmax
    st = lib.w8a8_gemm_silu(16, 16, 16, 16, None, 16, None, 4, 512, 256, None, 0, None)
    assert st == L.ERR_INVALID_ARG and b"amax" in lib.w8a8_last_error()
    assert lib.w8a8_gemm_silu(None, None, None, None, None, None, None, 0, 512, 256, None, 0, None) == L.OK
    st = lib.w8a8_quant_rows_amax(None, 16, None, None, None, 4, 16, None)
    assert st == L.ERR_INVALID_ARG and b"null" in lib.w8a8_last_error()
    st = lib.w8a8_quant_rows_amax(16, 16, 16, 16, 16, 4, 12, None)
    assert st == L.ERR_INVALID_ARG and b"multiple of 8" in lib.w8a8_last_error()
    st = lib.w8a8_quant_rows_amax(24, 16, 16, 16, 16, 4, 16, None)
    assert st == L.ERR_ALIGNMENT
    assert lib.w8a8_quant_rows_amax(None, 16, None, None, None, 0, 16, None) == L.OK
    # broadcast / peak probe: rejected on the host
    assert lib.w8a8_broadcast(None, 16, 16, 0, None) == L.ERR_INVALID_ARG
    assert lib.w8a8_mma_peak_probe(2, 10, None, None) == L.ERR_INVALID_ARG


@pytest.mark.parametrize("m,n,k,variant,bn,swap", [
    (1, 24576, 4096, 3, 16, 1), (16, 24576, 4096, 3, 16, 1), (17, 24576, 4096, 4, 32, 1),
    (64, 6144, 1024, 5, 64, 1), (65, 6144, 1024, 2, 128, 0), (256, 5120, 8192, 2, 128, 0),
    (8192, 24576, 4096, 7, 256, 0), (8192, 4096, 12288, 7, 256, 0), (4096, 6400, 5120, 7, 256, 0),
    (4096, 1280, 8192, 7, 256, 0), (512, 5120, 1024, 7, 256, 0), (8192, 1280, 8192, 7, 256, 0),
    # too few 256 x 256 blocks to occupy half of the SM pairs: 1-SM tiles + stream-K
    (300, 1280, 5120, 2, 128, 0), (1024, 256, 4096, 2, 128, 0),
])
def test_planner_variant_choice(pkg, m, n, k, variant, bn, swap):
    p = pkg.ops.gemm_plan(m, n, k)
    assert (p["variant"], p["bn"], p["swap"]) == (variant, bn, swap)
    assert 1 <= p["grid"] <= 148
    assert p["kblocks"] == (k + 127) // 128
    assert p["gran"] in (1, p["kblocks"])
    if p["workspace_bytes"]:
        # stream-K: two int32 tile slots per CTA; pair variant: one 128 x 256 slot per CTA
        slots = 1 if p["variant"] == 7 else 2
        assert p["workspace_bytes"] >= slots * p["grid"] * 128 * p["bn"] * 4


def _schedule(tiles, kblocks, grid, gran=1):
    """Host model of the kernel's hybrid schedule (FragmentWalk, sk_begin,
    sk_owner): whole tiles dealt in grid-stride order, then stream-K ranges
    over the remaining tiles' k blocks.  With a remainder and a full wave, the
    last full wave joins the stream-K part (two-tile stream-K).  Returns
    per-CTA fragment lists."""
    full, rem = divmod(tiles, grid)
    dp = (full - 1 if rem and full >= 1 else full) * grid
    units = (tiles - dp) * kblocks // gran
    sk = max(1, min(grid, units))            # CTAs sharing the stream-K part
    begin = [dp * kblocks + (min(c, sk) * units // sk) * gran for c in range(grid + 1)]
    owner = lambda x: (((x - dp * kblocks) // gran + 1) * sk - 1) // units  # noqa: E731
    frags = []
    for c in range(grid):
        f = [(t, 0, kblocks) for t in range(c, dp, grid)]
        it, end = begin[c], begin[c + 1]
        while it < end:
            t, k0 = divmod(it, kblocks)
            k1 = min(kblocks, k0 + (end - it))
            f.append((t, k0, k1))
            it += k1 - k0
        frags.append(f)
    return frags, begin, owner


@pytest.mark.parametrize("tiles,kblocks,grid", [(400, 40, 148), (32, 96, 148), (7, 3, 5), (6400, 40, 148),
                                                (80, 40, 148), (3, 1, 3), (1, 1, 1), (200, 7, 64),
                                                (119, 9, 148), (296, 40, 148), (160, 4, 148),
                                                (150, 2, 148), (149, 1, 148), (300, 3, 148)])
def test_hybrid_schedule_covers_every_iteration_once(tiles, kblocks, grid):
    grid = min(grid, tiles * kblocks)
    frags, begin, owner = _schedule(tiles, kblocks, grid)
    seen = {}
    for c, f in enumerate(frags):
        for (t, k0, k1) in f:
            for k in range(k0, k1):
                assert (t, k) not in seen
                seen[(t, k)] = c
    assert len(seen) == tiles * kblocks
    # per cut tile: the owners of its first and last iteration bound its
    # fragments, and the workspace slots (2c + started-before-tile) are distinct
    for t in range(tiles):
        owners = sorted({seen[(t, k)] for k in range(kblocks)})
        if len(owners) == 1:
            continue
        c0, c1 = owner(t * kblocks), owner(t * kblocks + kblocks - 1)
        assert owners == list(range(c0, c1 + 1))
        if tiles >= grid:  # two-tile stream-K: a tile is cut between at most two CTAs
            assert len(owners) <= 2
        slots = {2 * c + (1 if begin[c] < t * kblocks else 0) for c in owners}
        assert len(slots) == len(owners)
    # every stream-K CTA has work, and k blocks per CTA differ by at most one
    # tile when the remainder is smaller than the grid, else by at most one
    work = [sum(k1 - k0 for _, k0, k1 in f) for f in frags]
    assert max(work) - min(work) <= max(1, kblocks if (tiles % grid) * kblocks < grid else 1)


def test_hybrid_schedule_randomized_sweep():
    """The same invariants over a seeded sweep of (tiles, k blocks, grid):
    every iteration once; a cut tile's CTAs are contiguous with distinct
    workspace slots; at most two CTAs per tile once there is a full wave."""
    import random

    rng = random.Random(1234)
    for _ in range(300):
        grid = rng.choice([1, 2, 3, 7, 16, 64, 74, 128, 148])
        tiles = rng.randint(1, 6 * grid + 5)
        kblocks = rng.randint(1, 64)
        grid = min(grid, tiles * kblocks)
        frags, begin, owner = _schedule(tiles, kblocks, grid)
        seen = {}
        for c, f in enumerate(frags):
            for (t, k0, k1) in f:
                for k in range(k0, k1):
                    assert (t, k) not in seen
                    seen[(t, k)] = c
        assert len(seen) == tiles * kblocks, (tiles, kblocks, grid)
        for t in range(tiles):
            owners = sorted({seen[(t, k)] for k in range(kblocks)})
            if len(owners) == 1:
                continue
            assert owners == list(range(owners[0], owners[-1] + 1))
            assert (owner(t * kblocks), owner(t * kblocks + kblocks - 1)) == (owners[0], owners[-1])
            if tiles >= grid:
                assert len(owners) <= 2, (tiles, kblocks, grid, t)
            slots = {2 * c + (1 if begin[c] < t * kblocks else 0) for c in owners}
            assert len(slots) == len(owners)


def test_planner_stream_k_balances_few_tiles(pkg):
    # decode: down_proj of the Qwen3-8B MLP has only 32 weight tiles; stream-K
    # still spreads its 3072 k-block iterations over every SM
    p = pkg.ops.gemm_plan(1, 4096, 12288)
    assert p["tiles"] == 32 and p["grid"] == 148 and p["gran"] == 1 and p["workspace_bytes"] > 0
    # a prefill shape whose iterations split evenly into whole tiles needs no workspace
    p = pkg.ops.gemm_plan(8192, 24576, 4096, variant=1, ctas=128)
    assert p["grid"] == 128 and p["workspace_bytes"] == 0
    # the pair variant deals whole 256 x 256 blocks to an even number of CTAs
    p = pkg.ops.gemm_plan(8192, 24576, 4096)
    assert p["variant"] == 7 and p["grid"] == 148 and p["workspace_bytes"] == 0


def _pair_split(pairs, clusters, kblocks):
    """Host model of the pair variant's last-wave K split (plan_gemm): a last
    wave at most half full goes to min(clusters // rem, 4) pairs per block,
    each with at least 8 k blocks."""
    rem = pairs % clusters
    if pairs < clusters or rem == 0 or 2 * rem > clusters:
        return 0
    split = min(clusters // rem, 4)
    while split > 1 and kblocks // split < 8:
        split -= 1
    return split if split >= 2 else 0


@pytest.mark.parametrize("m,n,k,ctas", [
    (4096, 5120, 25600, 0), (4096, 5120, 8192, 0),       # 320 blocks on 74 pairs: 24 left, split 3
    (8192, 24576, 4096, 0),                              # 3072 blocks: 38 left, more than half a wave
    (1100, 1024, 2128, 16), (500, 1200, 4224, 18), (1280, 1024, 3200, 18), (1280, 1024, 2176, 12),
    (1280, 1024, 2176, 10),                              # 20 blocks on 5 pairs: no last wave
    (1280, 1024, 1024, 12),                              # 8 k blocks: shares would be under 8
])
def test_planner_pair_last_wave_split(pkg, m, n, k, ctas):
    p = pkg.ops.gemm_plan(m, n, k, variant=7, ctas=ctas, num_sms=148)
    pairs = ((m + 255) // 256) * ((n + 255) // 256)
    clusters = p["grid"] // 2
    split = _pair_split(pairs, clusters, (k + 127) // 128)
    if split:
        assert p["workspace_bytes"] == 256 * 1024 + p["grid"] * 128 * 256 * 4
    else:
        assert p["workspace_bytes"] == 0
    # a workspace too small for the slots keeps whole blocks
    q = pkg.ops.gemm_plan(m, n, k, variant=7, ctas=ctas, num_sms=148, workspace_bytes=1 << 20)
    assert q["workspace_bytes"] == 0 and q["grid"] == p["grid"]
    if (m, n, k, ctas) == (4096, 5120, 25600, 0):
        assert split == 3


def _pair_walk(pairs, clusters, kblocks, split):
    """Host model of the pair kernel's PairWalk: cluster c takes whole blocks
    c, c + G, ... below full = pairs - rem, then (split > 1) fragment f = c of
    the last wave: block full + f // split, k blocks [j kb / split, (j + 1) kb
    / split) with j = f % split.  Returns {cluster: [(block, k0, k1, j)]}."""
    rem = pairs % clusters if split else 0
    full = pairs - rem
    walk = {}
    for c in range(clusters):
        items = [(b, 0, kblocks, -1) for b in range(c, full if split else pairs, clusters)]
        if split and c < rem * split:
            j = c % split
            items.append((full + c // split, j * kblocks // split, (j + 1) * kblocks // split, j))
        walk[c] = items
    return walk


@pytest.mark.parametrize("m,n,k,ctas", [
    (4096, 5120, 25600, 0), (4096, 5120, 8192, 0), (4096, 2560, 5120, 0), (4096, 1280, 5120, 0),
    (1100, 1024, 2128, 16), (500, 1200, 4224, 18), (1280, 1024, 3200, 18), (1280, 1024, 2176, 12),
    (8192, 1280, 8192, 0), (3000, 3000, 3000, 0),
])
def test_pair_walk_covers_every_k_block_once(pkg, m, n, k, ctas):
    """Every (block, k block) of the pair plan is computed exactly once; a
    split block's share 0 sits on the pair whose next split - 1 pairs hold
    shares 1.. of the same block (the owner protocol's slot addressing), and
    every share has at least 8 k blocks."""
    p = pkg.ops.gemm_plan(m, n, k, variant=7, ctas=ctas, num_sms=148)
    pairs = ((m + 255) // 256) * ((n + 255) // 256)
    clusters = p["grid"] // 2
    kb = (k + 127) // 128
    split = _pair_split(pairs, clusters, kb)
    walk = _pair_walk(pairs, clusters, kb, split)
    seen = {}
    for c, items in walk.items():
        for b, k0, k1, j in items:
            for x in range(k0, k1):
                assert (b, x) not in seen, (b, x)
                seen[(b, x)] = c
            if j == 0:
                for o in range(1, split):
                    b2, k0b, k1b, j2 = walk[c + o][-1]
                    assert (b2, j2) == (b, o) and k0b == (o * kb) // split
            if j >= 0:
                assert k1 - k0 >= 8
    assert len(seen) == pairs * kb


def test_every_plan_fits_the_static_scratch(pkg):
    """The no-allocation entry point's 20 MiB scratch covers every stream-K plan
    the planner makes on a 148-SM device (the largest, 128 x 128 tiles with a
    cut remainder, needs 256 KiB of counters + 2 x 148 x 64 KiB)."""
    worst = 0
    for m in (1, 16, 17, 32, 33, 64, 65, 100, 128, 129, 200, 256, 300, 512, 1024, 4096, 8192):
        for n in (256, 1280, 2560, 5120, 6400, 10240, 25600, 51200):
            for k in (512, 1024, 5120, 8192, 25600):
                worst = max(worst, pkg.ops.gemm_plan(m, n, k, num_sms=148)["workspace_bytes"])
    assert worst == 256 * 1024 + 2 * 148 * 128 * 128 * 4
    assert worst <= 20 * 2 ** 20


def test_planner_respects_workspace_limit(pkg):
    p = pkg.ops.gemm_plan(1, 4096, 12288, workspace_bytes=0)
    assert p["gran"] == p["kblocks"] and p["workspace_bytes"] == 0 and p["grid"] == 32
    p = pkg.ops.gemm_plan(1, 4096, 12288, ctas=7)
    assert p["grid"] == 7 and p["gran"] == 1
    with pytest.raises(pkg.W8A8Error):
        pkg.ops.gemm_plan(1, 4096, 12288, ctas=-1)


def test_ops_refuse_cpu_tensors(pkg):
    import torch

    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    with pytest.raises(pkg.W8A8Error, match="no CPU path"):
        pkg.ops.quant_per_token(x)
    with pytest.raises(pkg.W8A8Error, match="no CPU path"):
        pkg.ops.w8a8_gemm(torch.zeros(4, 16, dtype=torch.int8), torch.zeros(16, 16, dtype=torch.int8),
                          torch.zeros(4), torch.zeros(16))


def test_gemm_operand_checks_run_on_the_host(pkg):
    """Both GEMM entries (plain and fused row-parallel) reject a short or
    mistyped scale vector and host (CPU) tensors before any pointer reaches
    the library; the fused entry needs no communicator buffers to do so."""
    import torch

    C = pkg.comm.PeerMemCommunicator
    comm = C.__new__(C)  # no device buffers: the checks come before any library call
    comm.device = torch.device("cuda", 0)
    a = torch.zeros(4, 32, dtype=torch.int8)
    w = torch.zeros(16, 32, dtype=torch.int8)
    for fn in (comm.gemm_allreduce, pkg.ops.w8a8_gemm):
        with pytest.raises(pkg.W8A8Error, match="shape mismatch"):
            fn(a, w, torch.ones(3), torch.ones(16))  # short activation scales
        with pytest.raises(pkg.W8A8Error, match="shape mismatch"):
            fn(a, w, torch.ones(4), torch.ones(8))  # short weight scales
        with pytest.raises(pkg.W8A8Error, match="fp32 scales"):
            fn(a, w, torch.ones(4, dtype=torch.float16), torch.ones(16))
        with pytest.raises(pkg.W8A8Error, match="bias"):
            fn(a, w, torch.ones(4), torch.ones(16), torch.ones(8, dtype=torch.bfloat16))
        with pytest.raises(pkg.W8A8Error, match="CUDA tensors required"):
            fn(a, w, torch.ones(4), torch.ones(16))  # host (CPU) weight and activations
