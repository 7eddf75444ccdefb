"""Activation quantiser feeding the hot path (kernels/norm.py:75-92 of the reference)."""
from .. import _lib


def quant_row(x, q, s):
    """bf16 x [M,K] -> int8 q [M,K], per-64-group fp32 scales s [M,K/64].

    ``s = max(amax / 127, 1e-8)``, ``q = round_half_away(x / s)`` clamped to
    +-127, with IEEE division (kernels/norm.py:15-25).  Returns ``(q, s)``.
    """
    rc = _lib.ext().quant_row(x, q, s)
    if rc:
        raise _lib.QlinError("qlin_quant_row", rc)
    return q, s
