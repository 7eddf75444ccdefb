"""Argument checks and pointer plumbing shared by the kernel shims.

The reference performs no validation (a bad shape is undefined behaviour in
its Triton kernels).  These shims reject what the CUDA path cannot honour
with ``ValueError`` / ``TypeError`` before anything is launched, and the C ABI
re-checks shapes and alignment (``QlinError`` on failure).
"""
import torch

from .. import _lib


def ptr(t):
    return None if t is None else t.data_ptr()


try:
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def stream_of(t):
    """Raw handle of torch's current CUDA stream on ``t``'s device."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def need(t, name, dtype, dims=None, contiguous=True):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path), got {t.device}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if dims is not None and t.dim() != dims:
        raise ValueError(f"{name} must be {dims}-D, got shape {tuple(t.shape)}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def need_rows(t, name, dtype):
    """2-D tensor whose rows may be strided but whose elements are contiguous."""
    need(t, name, dtype, 2, contiguous=False)
    if t.shape[1] > 1 and t.stride(1) != 1:
        raise ValueError(f"{name} must have unit stride along its last dimension")


def need_block_k(block_k):
    if block_k != 64:
        raise ValueError("block_k must equal GROUP (64): one activation scale per K block")


def call(fn_name, device, *args):
    """Invoke ``fn_name`` on ``device`` and raise ``QlinError`` on failure."""
    lib = _lib.load()
    fn = getattr(lib, fn_name)
    if device.index is not None and device.index != torch.cuda.current_device():
        with torch.cuda.device(device):
            rc = fn(*args)
    else:
        rc = fn(*args)
    _lib.check(fn_name, rc)
