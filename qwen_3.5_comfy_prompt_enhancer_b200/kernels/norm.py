"""Activation producers feeding the hot path -- drop-in for the reference's
``kernels/norm.py``: the same names, signatures, in-place outputs and return
values, backed by the sm_100a kernels of ``libqlin.so``.

Every producer writes int8 activations with one fp32 scale per 64-element
group (``s = max(amax / 127, 1e-8)``, ``q = round_half_away(y / s)`` clamped to
+-127, IEEE division; kernels/norm.py:15-25), except ``norm_gated`` (bf16) and
``gate_proj`` (the fp32 linear-attention gates).
"""
from .. import _lib


def _run(fn, rc):
    if rc:
        raise _lib.QlinError(fn, rc)


def quant_row(x, q, s):
    """bf16 x [M,K] -> int8 q [M,K], per-64-group fp32 scales s [M,K/64]
    (kernels/norm.py:75-92).  Returns ``(q, s)``."""
    _run("qlin_quant_row", _lib.ext().quant_row(x, q, s))
    return q, s


def rmsnorm_quant(x, w, q, s, eps=1e-6, one_plus=True):
    """x: bf16 [M,K] (row stride may differ), w: [K], q: int8 [M,K], s: fp32 [M,K/64]
    (kernels/norm.py:28-57): ``y = x * rsqrt(mean(x^2) + eps) * (1 + w)``
    (``w`` itself without ``one_plus``), quantised per 64.  Returns ``(q, s)``."""
    _run("qlin_rmsnorm_quant", _lib.ext().rmsnorm_quant(x, w, q, s, float(eps), bool(one_plus)))
    return q, s


def norm_gated_quant(v, z, w, q, s, eps=1e-6):
    """v: [T, NV*HD] bf16, z: [T, NV*HD] gate, w: [HD] (kernels/norm.py:95-137).
    Per (token, head): ``y = x * rsqrt(mean(x^2) + eps) * w * silu(z)``, rounded
    through bf16, quantised per 64 within the head into q int8 [T, NV*HD] and
    s fp32 [T, (NV*HD)//64].  Returns ``(q, s)``."""
    _run("qlin_norm_gated_quant", _lib.ext().norm_gated(v, z, w, q, s, None, float(eps)))
    return q, s


def norm_gated(v, z, w, out, eps=1e-6):
    """Gated RMSNorm of the delta-rule output stored as bf16 ``out``
    (kernels/norm.py:141-165).  Returns ``out``."""
    _run("qlin_norm_gated", _lib.ext().norm_gated(v, z, w, None, None, out, float(eps)))
    return out


def gate_mul_quant(a, g, q, s, hd=256):
    """out = a * sigmoid(G) with G laid out as [M, heads, 2*HD] (gate in the
    second half of each head), quantised per 64 (kernels/norm.py:168-188).
    Returns ``(q, s)``."""
    _run("qlin_gate_mul_quant", _lib.ext().gate_mul_quant(a, g, q, s, int(hd)))
    return q, s


def silu_mul_quant(g, u, q, s):
    """``silu(g) * u`` quantised per 64 (kernels/norm.py:191-208).  Returns ``(q, s)``."""
    _run("qlin_silu_mul_quant", _lib.ext().silu_mul_quant(g, u, q, s))
    return q, s


def gate_proj(a_q, a_s, wb, wa, beta, gate, dt_bias, a_log):
    """beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias), from int8
    activations (kernels/norm.py:211-240): ``b = wb @ (a_q * a_s)``,
    ``a = wa @ (a_q * a_s)`` per row.  Returns ``(beta, gate)``."""
    _run("qlin_gate_proj", _lib.ext().gate_proj(a_q, a_s, wb, wa, beta, gate, dt_bias, a_log))
    return beta, gate
