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
    assert pl["nbb"] * pl["bs"] * ns * nsub * nm <= TMEM_SHARE
    single = pl["bs"] == pl["gmax"]
    if single:
        assert (pl["rb"], pl["nbb"]) == (1, 1)
    else:
        assert pl["rb"] == 2 and pl["nbb"] == 2
    assert pl["ab"] == (0 if wbits == 8 else pl["rb"])


@pytest.mark.parametrize("wbits,gate_up,M,K,N,wgrp,split", [
    (8, 0, 1, 2048, 6144, 64, 4),      # config 1: W8 projection at decode
    (4, 1, 4, 2048, 6144, 128, 4),     # config 2: fused gate/up, 4 rows
    (4, 0, 4, 6144, 2048, 128, 8),     # config 2: down projection (K = 6144)
    (4, 0, 1, 2048, 2048, 128, 8),     # config 2: o projection
    (4, 0, 4, 2048, 4096, 128, 6),     # config 2: qkv + gate projection
])
def test_config_plans(pkg, wbits, gate_up, M, K, N, wgrp, split):
    pl = pkg._lib.plan_small_m(wbits, gate_up, M, K, tiles_of(N), wgrp, SMS)
    check_plan(pl, wbits, gate_up, M, K, wgrp)
    assert pl["split"] == split
    assert tiles_of(N) * pl["split"] <= (SMS * 4 + 2) // 3 or pl["split"] == 1


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
