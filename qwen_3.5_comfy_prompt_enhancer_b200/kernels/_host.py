"""Host helpers shared by the kernel shims.

The reference performs no validation (a bad shape is undefined behaviour in
its Triton kernels).  The entry points here check their tensors in the
compiled binding (``csrc/pyext.cpp``: dtype, rank, contiguity, shapes, one
CUDA device) and raise ``ValueError`` / ``TypeError`` before anything is
launched; the C ABI re-checks shapes and alignment (``QlinError`` on failure).
"""
import torch

try:
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def stream_of(t):
    """Raw handle of torch's current CUDA stream on ``t``'s device."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def need_block_k(block_k):
    if block_k != 64:
        raise ValueError("block_k must equal GROUP (64): one activation scale per K block")
