"""Activation quantiser feeding the hot path (kernels/norm.py:75-92 of the reference)."""
import torch

from ._host import call, need, need_rows, ptr, stream_of
from .common import GROUP


def quant_row(x, q, s):
    """bf16 x [M,K] -> int8 q [M,K], per-64-group fp32 scales s [M,K/64].

    ``s = max(amax / 127, 1e-8)``, ``q = round_half_away(x / s)`` clamped to
    +-127, with IEEE division (kernels/norm.py:15-25).  Returns ``(q, s)``.
    """
    need_rows(x, "x", torch.bfloat16)
    need(q, "q", torch.int8, 2)
    need(s, "s", torch.float32, 2)
    M, K = q.shape
    if tuple(x.shape) != (M, K) or tuple(s.shape) != (M, K // GROUP):
        raise ValueError(f"shapes must be x [M,K], q [M,K], s [M,K/64]; got {tuple(x.shape)}, "
                         f"{tuple(q.shape)}, {tuple(s.shape)}")
    call("qlin_quant_row", x.device, ptr(x), x.stride(0), M, K, ptr(q), ptr(s), stream_of(x))
    return q, s
