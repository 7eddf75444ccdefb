"""Fault path of the bounded device-side waits, exercised without faulting the
GPU.

A peer all-gather is launched as rank 0 of a world of two whose gather
buffers and arrival counters are all local allocations of this process; the
second "rank" never calls, so the arrival that rank 0 waits for never comes.
With the wait bound lowered to 50 ms the kernel gives up, records the fault
and returns; every access stays inside the buffers.  The test then checks that
the fault is reported: by the fault word, by QLIN_ERR_DEVICE_FAULT from the
next entry point (C ABI) and by QlinError (Python), and that clearing it
restores normal service.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O
from qlin_testutil import bits

pytestmark = pytest.mark.gpu

QLIN_ERR_DEVICE_FAULT = 6


def _ptrs(*tensors):
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


@pytest.fixture
def lib(pkg, dev):
    """The C ABI; the fault word is cleared again afterwards whatever happens,
    so that no later test sees this test's fault."""
    torch.cuda.set_device(dev)
    lib = pkg._lib.load()
    yield lib
    torch.cuda.synchronize()
    lib.qlin_set_wait_limit_ns(2_000_000_000)
    lib.qlin_device_fault(1)


def test_timed_out_wait_is_reported_and_cleared(pkg, dev, lib):
    stream = torch.cuda.current_stream(dev).cuda_stream
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(4, 256, device=dev, generator=g).to(torch.bfloat16)
    q = torch.empty(4, 256, dtype=torch.int8, device=dev)
    s = torch.empty(4, 4, dtype=torch.float32, device=dev)
    pkg.quant_row(x, q, s)            # sets up the host-visible fault mirror
    torch.cuda.synchronize()
    assert lib.qlin_device_fault(1) == 0

    n = 4096
    bufs = [torch.zeros(2 * n, dtype=torch.uint8, device=dev) for _ in range(2)]
    arrive = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
    expected = torch.zeros(2, dtype=torch.int32, device=dev)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g)
    assert lib.qlin_set_wait_limit_ns(50_000_000) == 0
    try:
        t0 = time.perf_counter()
        rc = lib.qlin_peer_allgather(_ptrs(*bufs), _ptrs(*arrive), expected.data_ptr(), src.data_ptr(), n, 2, 0,
                                     None, stream)
        assert rc == 0, lib.qlin_last_error()
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        assert lib.qlin_set_wait_limit_ns(2_000_000_000) == 0
    assert elapsed < 1.5, f"kernel returned after {elapsed:.2f} s, not after the 50 ms bound"
    # rank 0's shard reached slot 0 of both buffers and its arrival was counted;
    # rank 1's never came
    assert torch.equal(bufs[0][:n], src) and torch.equal(bufs[1][:n], src)
    assert arrive[0][0].item() == 1 and arrive[0][1].item() == 0
    fw = lib.qlin_device_fault(0)
    assert fw & 1, f"fault word {fw:#x}"

    # the next launch through the C ABI reports the earlier fault ...
    rc = lib.qlin_quant_row(x.data_ptr(), 256, 4, 256, q.data_ptr(), s.data_ptr(), stream)
    assert rc == QLIN_ERR_DEVICE_FAULT
    assert b"earlier launch" in lib.qlin_last_error()
    # ... and so does the Python layer
    with pytest.raises(pkg._lib.QlinError) as ei:
        pkg.quant_row(x, q, s)
    assert ei.value.status == QLIN_ERR_DEVICE_FAULT

    # clearing restores normal service
    assert lib.qlin_device_fault(1) & 1
    assert lib.qlin_device_fault(0) == 0
    pkg.quant_row(x, q, s)
    torch.cuda.synchronize()
    rq, rs = O.quant_row(bits(x))
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_flagged_word_gather_times_out_without_its_peer(pkg, dev, lib):
    """The column-split layer's gather (qlin_peer_allgather_ll) as rank 0 of
    two, both exchange buffers local: rank 1's words never come, so the
    receiving threads give up after the 50 ms bound and the fault is
    recorded; rank 0's own block still reached its slot of the destination
    and, as flagged words of call 1, rank 1's exchange buffer."""
    stream = torch.cuda.current_stream(dev).cuda_stream
    x = torch.randn(4, 256, device=dev).to(torch.bfloat16)
    q = torch.empty(4, 256, dtype=torch.int8, device=dev)
    s = torch.empty(4, 4, dtype=torch.float32, device=dev)
    pkg.quant_row(x, q, s)            # sets up the host-visible fault mirror
    torch.cuda.synchronize()
    assert lib.qlin_device_fault(1) == 0

    rows, rb = 4, 1024
    g = torch.Generator(device=dev).manual_seed(12)
    src = torch.randint(0, 256, (rows, rb), dtype=torch.uint8, device=dev, generator=g)
    parts = (pkg._lib.GatherPart * 1)(pkg._lib.GatherPart(src.data_ptr(), rb, rows, rb, 0, 2 * rb))
    need = ctypes.c_int64()
    assert lib.qlin_peer_ll_bytes(parts, 1, 2, ctypes.byref(need)) == 0
    assert need.value == 2 * 2 * (rows * rb * 2)
    ll = [torch.zeros(need.value, dtype=torch.uint8, device=dev) for _ in range(2)]
    state = torch.zeros(16, dtype=torch.int32, device=dev)
    dst = torch.zeros(rows, 2 * rb, dtype=torch.uint8, device=dev)
    assert lib.qlin_set_wait_limit_ns(50_000_000) == 0
    try:
        t0 = time.perf_counter()
        rc = lib.qlin_peer_allgather_ll(_ptrs(*ll), need.value, state.data_ptr(), parts, 1, 2, 0,
                                        dst.data_ptr(), stream)
        assert rc == 0, lib.qlin_last_error()
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        assert lib.qlin_set_wait_limit_ns(2_000_000_000) == 0
    assert elapsed < 1.5, f"kernel returned after {elapsed:.2f} s, not after the 50 ms bound"
    assert torch.equal(dst[:, :rb], src)
    assert not dst[:, rb:].any()      # rank 1's slot: nothing came
    # call 1 uses the odd half; rank 0's slot of rank 1's buffer holds words (1 << 32 | data)
    words = ll[1].cpu().numpy().view(np.uint64)[need.value // 16: need.value // 16 + rows * rb // 4]
    np.testing.assert_array_equal(words >> np.uint64(32), np.ones(rows * rb // 4, dtype=np.uint64))
    np.testing.assert_array_equal((words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.uint8).reshape(rows, rb),
                                  src.cpu().numpy())
    assert state[0].item() == 1       # the call still completed and counted itself
    assert lib.qlin_device_fault(0) & 1
    rc = lib.qlin_quant_row(x.data_ptr(), 256, 4, 256, q.data_ptr(), s.data_ptr(), stream)
    assert rc == QLIN_ERR_DEVICE_FAULT
    assert lib.qlin_device_fault(1) & 1
    assert lib.qlin_device_fault(0) == 0


def test_fused_down_projection_times_out_without_its_peer(pkg, dev, lib):
    """The column-split down projection with the gathers inside
    (qlin_tp_gemm_w4_ll) as rank 0 of two, every buffer local: rank 0's h
    words are sent, rank 1's never, so the CTAs whose K part lies in rank 1's
    columns give up polling after the 50 ms bound and record the fault; the
    launch returns and a clear restores service."""
    stream = torch.cuda.current_stream(dev).cuda_stream
    x = torch.randn(4, 256, device=dev).to(torch.bfloat16)
    q = torch.empty(4, 256, dtype=torch.int8, device=dev)
    s = torch.empty(4, 4, dtype=torch.float32, device=dev)
    pkg.quant_row(x, q, s)            # sets up the host-visible fault mirror
    torch.cuda.synchronize()
    assert lib.qlin_device_fault(1) == 0

    M, K, N, WG, world = 1, 4096, 640, 128, 2
    kloc = K // world
    g = torch.Generator(device=dev).manual_seed(13)
    b = torch.randint(0, 256, (K // 2, N), dtype=torch.uint8, device=dev, generator=g)
    sc = torch.full((K // WG, N), 0.01, dtype=torch.bfloat16, device=dev)
    hq_loc = torch.randint(-127, 128, (M, kloc), dtype=torch.int8, device=dev, generator=g)
    hs_loc = torch.full((M, kloc // 64), 0.01, dtype=torch.float32, device=dev)
    slot = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    P = pkg._lib.GatherPart
    hs_off = K  # codes [M, K] then scales
    h_arr = (P * 2)(P(hq_loc.data_ptr(), kloc, M, kloc, 0, K), P(hs_loc.data_ptr(), kloc // 16, M, kloc // 16, hs_off, K // 16))
    o_arr = (P * 1)(P(slot.data_ptr(), 2 * N, M, 2 * N, 0, 2 * N))
    hb, ob = ctypes.c_int64(), ctypes.c_int64()
    assert lib.qlin_peer_ll_bytes(h_arr, 2, world, ctypes.byref(hb)) == 0
    assert lib.qlin_peer_ll_bytes(o_arr, 1, world, ctypes.byref(ob)) == 0
    h_ll = [torch.zeros(hb.value, dtype=torch.uint8, device=dev) for _ in range(world)]
    o_ll = [torch.zeros(ob.value, dtype=torch.uint8, device=dev) for _ in range(world)]
    h_state = torch.zeros(16, dtype=torch.int32, device=dev)
    o_state = torch.zeros(16, dtype=torch.int32, device=dev)
    plan = (ctypes.c_int64 * 4)()
    assert lib.qlin_plan_dp(4, 0, M, K, N // 128, WG, 0, plan) == 0 and plan[0] > 0
    assert lib.qlin_set_wait_limit_ns(50_000_000) == 0
    try:
        t0 = time.perf_counter()
        assert lib.qlin_peer_ll_send(_ptrs(*h_ll), hb.value, h_state.data_ptr(), h_arr, 2, world, 0, stream) == 0
        rc = lib.qlin_tp_gemm_w4_ll(M, K, b.data_ptr(), sc.data_ptr(), None, N, WG, slot.data_ptr(), N,
                                    _ptrs(*h_ll), hb.value, h_state.data_ptr(), h_arr, 2, _ptrs(*o_ll), ob.value,
                                    o_state.data_ptr(), o_arr, 1, world, 0, None, None, stream)
        assert rc == 0, lib.qlin_last_error()
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        assert lib.qlin_set_wait_limit_ns(2_000_000_000) == 0
    assert elapsed < 1.5, f"kernel returned after {elapsed:.2f} s, not after the 50 ms bound"
    assert lib.qlin_device_fault(0) & 1
    rc = lib.qlin_quant_row(x.data_ptr(), 256, 4, 256, q.data_ptr(), s.data_ptr(), stream)
    assert rc == QLIN_ERR_DEVICE_FAULT
    assert lib.qlin_device_fault(1) & 1
    assert lib.qlin_device_fault(0) == 0
    pkg.quant_row(x, q, s)
    torch.cuda.synchronize()
