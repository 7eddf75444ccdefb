"""The all-gather that allocates nothing (``qlin_peer_allgather_static``),
called through the C ABI and checked byte for byte against its input (at
world = 1 the gathered bytes are the shard itself) and against the allocating
``qlin_peer_allgather`` (world = 1) on the same shards.

It is for a process that runs the column-split layer on one GPU and may not
call cudaMalloc itself -- a plugin whose host application owns all device
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


def test_static_gather_matches_allocating_gather_in_a_row(pkg):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = pkg._lib.load()
    g = torch.Generator(device=dev).manual_seed(7)
    shards = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g)
              for n in (96 * 1024, 96 * 1024, 4096, LIMIT)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    outs = [torch.empty_like(s) for s in shards]
    for s, o in zip(shards, outs):  # back to back, no synchronisation in between
        rc = lib.qlin_peer_allgather_static(s.data_ptr(), s.numel(), o.data_ptr(), stream)
        assert rc == 0, lib.qlin_last_error()
    refs = [_existing_gather(lib, s, dev) for s in shards]
    torch.cuda.synchronize()
    for s, o, r in zip(shards, outs, refs):
        assert torch.equal(o, s)   # world 1: the gathered bytes are the shard itself
        assert torch.equal(o, r)
    assert lib.qlin_device_fault(1) == 0


def test_static_gather_rejects_sizes_beyond_its_limit(pkg):
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    lib = pkg._lib.load()
    src = torch.zeros(LIMIT + 16, dtype=torch.uint8, device=dev)
    out = torch.empty_like(src)
    rc = lib.qlin_peer_allgather_static(src.data_ptr(), src.numel(), out.data_ptr(),
                                        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 2 and b"limit" in lib.qlin_last_error()
