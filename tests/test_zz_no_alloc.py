"""The all-gather that allocates nothing (``qlin_peer_allgather_static``),
called through the C ABI and checked byte for byte against the allocating
``qlin_peer_allgather`` on the same shards.

It is for programs that drive every rank's GPU from one process and may not
call cudaMalloc themselves -- a plugin whose host application owns all device
memory through its own pool, say.  Its buffer and counters are static device
arrays of the library, shared by every call, so the tests below make several
calls in a row.  This file is named to be collected last: if it fails, a run
that stops at the first failure has run every other test already.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT = 4 << 20  # QLIN_STATIC_GATHER_MAX_BYTES


def _ptrs(*tensors):
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


def _existing_gather(lib, src, dev):
    """World-1 all-gather through the allocating entry point (caller-owned buffers)."""
    n = src.numel()
    buf = torch.zeros(n, dtype=torch.uint8, device=dev)
    arrive = torch.zeros(1, dtype=torch.int32, device=dev)
    expected = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    rc = lib.qlin_peer_allgather(_ptrs(buf), _ptrs(arrive), expected.data_ptr(), src.data_ptr(), n, 1, 0,
                                 out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, lib.qlin_last_error()
    return out


def test_static_gather_matches_allocating_gather_twice(pkg):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = pkg._lib.load()
    g = torch.Generator(device=dev).manual_seed(7)
    shards = [torch.randint(0, 256, (96 * 1024,), dtype=torch.uint8, device=dev, generator=g) for _ in range(3)]
    devices = (ctypes.c_int * 1)(0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    outs = [torch.empty_like(s) for s in shards]
    for s, o in zip(shards, outs):  # back to back, no synchronisation in between
        rc = lib.qlin_peer_allgather_static(devices, 1, 0, s.data_ptr(), s.numel(), o.data_ptr(), stream)
        assert rc == 0, lib.qlin_last_error()
    refs = [_existing_gather(lib, s, dev) for s in shards]
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    assert lib.qlin_device_fault(1) == 0


def test_static_gather_rejects_sizes_beyond_its_limit(pkg):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = pkg._lib.load()
    src = torch.zeros(LIMIT + 16, dtype=torch.uint8, device=dev)
    out = torch.empty_like(src)
    devices = (ctypes.c_int * 1)(0)
    rc = lib.qlin_peer_allgather_static(devices, 1, 0, src.data_ptr(), src.numel(), out.data_ptr(),
                                        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 2 and b"limit" in lib.qlin_last_error()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_static_gather_two_gpus_one_process(pkg):
    """Two ranks on two GPUs of this process, twice in a row."""
    lib = pkg._lib.load()
    devs = [torch.device("cuda", i) for i in range(2)]
    devices = (ctypes.c_int * 2)(0, 1)
    n = 64 * 1024
    for call in range(2):
        srcs, outs = [], []
        for d in devs:
            g = torch.Generator(device=d).manual_seed(100 * call + d.index)
            srcs.append(torch.randint(0, 256, (n,), dtype=torch.uint8, device=d, generator=g))
            outs.append(torch.empty(2 * n, dtype=torch.uint8, device=d))
        for rank, d in enumerate(devs):  # both launches queued before either is waited on
            with torch.cuda.device(d):
                rc = lib.qlin_peer_allgather_static(devices, 2, rank, srcs[rank].data_ptr(), n,
                                                    outs[rank].data_ptr(), torch.cuda.current_stream(d).cuda_stream)
                assert rc == 0, lib.qlin_last_error()
        for d in devs:
            torch.cuda.synchronize(d)
        want = torch.cat([srcs[0].cpu(), srcs[1].cpu()])
        for o in outs:
            assert torch.equal(o.cpu(), want)
    for d in devs:
        with torch.cuda.device(d):
            assert lib.qlin_device_fault(1) == 0
