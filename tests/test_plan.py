"""Launch plans of the small-M tensor-core kernel, checked on the CPU.

``qlin_plan_small_m`` runs the same planner the entry points use, without a
GPU.  Every plan must fit one CTA's shared memory and tensor-memory share,
cover the whole K range, and keep the combine buffers bounded; the
config shapes must get the splits the planner documents."""
import itertools

import pytest

SMS = 148
MAX_SMEM = 227 * 1024
TMEM_SHARE = 256


def tiles_of(n):
    return (n + 127) // 128


def check_plan(pl, wbits, gate_up, M, K, wgrp):
    G = K // 64
    assert 1 <= pl["split"] <= 8
    assert pl["gmax"] * pl["split"] >= G
    assert pl["gmax"] == -(-G // pl["split"])
    assert 1 <= pl["bs"] <= pl["gmax"]
    assert pl["smem"] <= MAX_SMEM
    assert pl["mr"] in (1, 2, 4, 8, 16, 32)
    if wbits == 4:
        assert pl["mr"] <= 16
    nm = max(pl["mr"], 16)
    ns = 2 if gate_up else 1
    nsub = 2 if (wbits == 4 and wgrp == 32) else 1
    per_buf = ns * nsub * nm
    assert pl["nbb"] * pl["bs"] * per_buf <= TMEM_SHARE
    single = pl["bs"] == pl["gmax"] and pl["rb"] == 1
    if single:
        assert pl["nbb"] == 1 and pl["ab"] == (1 if wbits == 4 else 0)
    else:
        assert pl["rb"] in (2, 3, 4) and pl["nbb"] == 2 and pl["ab"] == (2 if wbits == 4 else 0)
    assert pl["level"] == (2 if single else 0)
    if pl["alias"]:
        # the partial sums of ranks 1..split-1 fit rank 0's operand region:
        # W4 ring tiles of 32 rows (high nibbles, groups of 64 k) or 64 rows
        # (both nibbles, groups of 32); W8 weight tiles of 64 rows
        assert pl["split"] >= 2 and pl["level"] == 2
        part = (pl["split"] - 1) * ns * pl["mr"] * 128 * 4
        rows = (64 if wgrp == 32 else 32) if wbits == 4 else 64
        op = (pl["ab"] if wbits == 4 else pl["rb"]) * pl["bs"] * ns * rows * 128
        assert part <= op


@pytest.mark.parametrize("wbits,gate_up,M,K,N,wgrp,split,level", [
    (8, 0, 1, 2048, 6144, 64, 4, 2),      # config 1: W8 projection at decode, one batch
    (4, 1, 4, 2048, 6144, 128, 4, 0),     # config 2: fused gate/up, streamed within the CTA target
    (4, 1, 1, 2048, 6144, 128, 4, 0),
    (4, 0, 4, 6144, 2048, 128, 8, 0),     # config 2: down projection (K = 6144), streamed
    (4, 0, 1, 2048, 2048, 128, 6, 2),     # config 2: o projection, compact one-batch plan
    (4, 0, 4, 2048, 4096, 128, 4, 2),     # config 2: qkv + gate projection, compact one-batch plan
])
def test_config_plans(pkg, wbits, gate_up, M, K, N, wgrp, split, level):
    pl = pkg._lib.plan_small_m(wbits, gate_up, M, K, tiles_of(N), wgrp, SMS)
    check_plan(pl, wbits, gate_up, M, K, wgrp)
    assert (pl["split"], pl["level"]) == (split, level)
    assert tiles_of(N) * pl["split"] <= 2 * SMS


@pytest.mark.parametrize("wbits,gate_up", [(8, 0), (8, 1), (4, 0), (4, 1)])
def test_plan_sweep_fits(pkg, wbits, gate_up):
    groups = (32, 64, 128, 256) if wbits == 4 else (64,)
    Ms = (1, 2, 3, 4, 5, 8, 11, 16, 17, 32, 37, 64, 100)
    Ks = (64, 128, 192, 1024, 2048, 2560, 4096, 6144, 9216, 12288, 17408, 25600)
    Ns = (16, 128, 1024, 2048, 6144, 17408, 151936)
    for wgrp, M, K, N in itertools.product(groups, Ms, Ks, Ns):
        if K % wgrp:
            continue
        pl = pkg._lib.plan_small_m(wbits, gate_up, M, K, tiles_of(N), wgrp, SMS)
        check_plan(pl, wbits, gate_up, M, K, wgrp)


def test_forced_split_never_oversized(pkg):
    # 32-row blocks with the largest K fall back to 16-row blocks rather than
    # exceed shared memory.
    pl = pkg._lib.plan_small_m(8, 1, 37, 17408, 48, 64, SMS)
    check_plan(pl, 8, 1, 37, 17408, 64)
    assert pl["mr"] == 16


def test_plan_rejects_bad_query(pkg):
    with pytest.raises(pkg._lib.QlinError):
        pkg._lib.plan_small_m(5, 0, 1, 2048, 16, 64, SMS)
    with pytest.raises(pkg._lib.QlinError):
        pkg._lib.plan_small_m(8, 0, 1, 100, 16, 64, SMS)
    with pytest.raises(pkg._lib.QlinError):
        pkg._lib.plan_small_m(4, 0, 1, 2048, 16, 48, SMS)


@pytest.mark.gpu
def test_cluster_capacity_query(pkg):
    """qlin_max_active_clusters answers on a GPU, never grows with the cluster
    size, and never exceeds the SM count divided by the cluster size."""
    import ctypes
    import torch
    torch.zeros(1, device="cuda:0")
    lib = pkg._lib.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    out = ctypes.c_int64()
    prev = None
    for split in range(1, 9):
        assert lib.qlin_max_active_clusters(4, 1, 4, split, 100 * 1024, ctypes.byref(out)) == 0
        assert 1 <= out.value <= sms // split
        if prev is not None:
            assert out.value <= prev
        prev = out.value


@pytest.mark.gpu
@pytest.mark.parametrize("gate_up,M,K,N", [
    (1, 1, 5120, 17408), (1, 4, 5120, 17408),       # config 5 gate/up on 1 GPU
    (0, 1, 17408, 5120), (0, 4, 17408, 5120),       # config 5 down on 1 GPU
    (0, 1, 17408, 2560), (1, 1, 5120, 4352),        # per-rank shapes of the 2- and 4-way splits
])
def test_launch_plans_fit_one_wave_of_clusters(pkg, gate_up, M, K, N):
    """On the device, the chosen plan's clusters are resident at once when any
    split allows that (the planner ranks second-wave plans last)."""
    import ctypes
    import torch
    torch.zeros(1, device="cuda:0")
    lib = pkg._lib.load()
    pl = pkg._lib.plan_small_m(4, gate_up, M, K, tiles_of(N), 128, 0)
    check_plan(pl, 4, gate_up, M, K, 128)
    out = ctypes.c_int64()
    assert lib.qlin_max_active_clusters(4, gate_up, M, pl["split"], pl["smem"], ctypes.byref(out)) == 0
    per_sm = min(2, (228 * 1024) // (pl["smem"] + 1024))
    cap = out.value
    if per_sm >= 2:  # the query counts one CTA per SM; the planner's estimate for two per SM
        s = pl["split"]
        c = lambda x: (lib.qlin_max_active_clusters(4, gate_up, M, x, pl["smem"], ctypes.byref(out)), out.value)[1]
        cap = 2 * c(1) if s == 1 else c(s // 2) if s % 2 == 0 else (c((s - 1) // 2) + c((s + 1) // 2)) // 2
    assert tiles_of(N) <= cap, (pl, cap)


def _plan_dp(pkg, wbits, gate_up, M, K, N, wgrp=128):
    import ctypes
    out = (ctypes.c_int64 * 4)()
    assert pkg._lib.load().qlin_plan_dp(wbits, gate_up, M, K, tiles_of(N), wgrp, SMS, out) == 0
    return list(out)


def test_decode_row_plans(pkg):
    """qlin_plan_dp (no GPU needed with an SM count): the decode-row launches
    of configs 1, 2 and 5 get the plans their profiles show, every plan covers
    K, and more than four rows go to the tensor-core kernels."""
    assert _plan_dp(pkg, 4, 1, 1, 2048, 6144)[:3] == [4, 1, 0]   # config-2 gate/up M = 1: resident, clusters of 4
    assert _plan_dp(pkg, 4, 1, 4, 2048, 6144)[:3] == [4, 1, 0]   # and M = 4
    assert _plan_dp(pkg, 8, 0, 1, 2048, 6144)[:3] == [4, 1, 0]   # config-1 W8
    split, kout, ring, _ = _plan_dp(pkg, 4, 0, 1, 17408, 640)    # config-5 8-GPU down shard: ring + K parts
    assert split == 1 and kout > 1 and ring > 0
    split, kout, ring, _ = _plan_dp(pkg, 4, 0, 1, 17408, 5120)   # config-5 down on one GPU: (1, 40, 7) grid
    assert (split, kout) == (1, 7) and ring > 0
    assert _plan_dp(pkg, 4, 0, 8, 2048, 2048) == [0, 0, 0, 0]
    for wbits, gate_up, M, K, N in itertools.product((4, 8), (0, 1), (1, 2, 3, 4), (2048, 5120, 6144, 17408),
                                                     (640, 2048, 6144, 17408)):
        split, kout, ring, gmax = _plan_dp(pkg, wbits, gate_up, M, K, N)
        if split:
            assert split * kout * gmax >= K // 64 and split <= 8


def test_flagged_word_exchange_size(pkg):
    """qlin_peer_ll_bytes: two halves x world senders x (two 8-byte words per 8
    data bytes, or per 4 data bytes where rows are not a multiple of 8), each
    part padded to 16 bytes."""
    import ctypes
    P = pkg._lib.GatherPart
    lib = pkg._lib.load()
    parts = (P * 2)(P(0, 2176, 4, 2176, 0, 8 * 2176), P(0, 36, 4, 36, 99999 * 8, 8 * 36))
    need = ctypes.c_int64()
    assert lib.qlin_peer_ll_bytes(parts, 2, 8, ctypes.byref(need)) == 0
    slot = 4 * 2176 * 2 + -(-(4 * 36 // 4) * 8 // 16) * 16
    assert need.value == 2 * 8 * slot
    assert lib.qlin_peer_ll_bytes(parts, 2, 9, ctypes.byref(need)) != 0   # more ranks than the kernels serve
