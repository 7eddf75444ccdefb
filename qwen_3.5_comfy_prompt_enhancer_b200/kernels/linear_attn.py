"""Gated delta-net (linear attention) decode neighbours -- drop-in for the
reference's ``kernels/linear_attn.py`` (``conv_silu``, ``conv_state_update``,
``delta_decode``), backed by the sm_100a kernels of ``libqlin.so``.
Head sizes are the reference's: NH = 16, DK = DV = 128 (linear_attn.py:203).
"""
from .. import _lib


def conv_silu(x, w, state, y, T, batch=False):
    """Depthwise causal conv (width 4) + SiLU (kernels/linear_attn.py:10-47).
    Returns ``y``."""
    rc = _lib.ext().conv_silu(x, w, state, y, int(T), bool(batch))
    if rc:
        raise _lib.QlinError("qlin_conv_silu", rc)
    return y


def conv_state_update(x, state, T, batch=1):
    """Shift the conv window: the state keeps the last 3 raw input rows
    (kernels/linear_attn.py:50-83)."""
    rc = _lib.ext().conv_state_update(x, state, int(T), int(batch))
    if rc:
        raise _lib.QlinError("qlin_conv_state_update", rc)


def delta_decode(qkv, g, beta, state, out, vs=32, batch=1):
    """One recurrent delta-rule step per batch row (kernels/linear_attn.py:172-207);
    ``state`` [batch*NH, DK, DV] fp32 is updated in place.  ``vs`` is accepted
    and ignored.  Returns ``out``."""
    rc = _lib.ext().delta_decode(qkv, g, beta, state, out, int(batch))
    if rc:
        raise _lib.QlinError("qlin_delta_decode", rc)
    return out


def delta_prefill(qkv, g, beta, state, out, T, vs=32, chunk=32):
    """Chunked (32-token) gated delta rule over T tokens (kernels/linear_attn.py:98-169);
    ``state`` [NH, DK, DV] fp32 is updated in place.  ``vs`` / ``chunk`` are
    accepted and ignored (the kernel's own tiling; the chunk is 32).
    Returns ``out``."""
    rc = _lib.ext().delta_prefill(qkv, g, beta, state, out, int(T))
    if rc:
        raise _lib.QlinError("qlin_delta_prefill", rc)
    return out


def conv_silu_update(x, w, state, y, batch):
    """``conv_silu(x, w, state, y, batch, batch=True)`` followed by
    ``conv_state_update(x, state, batch, batch=batch)`` in one launch (one
    decode row per candidate); identical results.  Not in the reference,
    whose engine makes the two calls back to back (engine.py:302-303).
    Returns ``y``."""
    rc = _lib.ext().conv_silu_update(x, w, state, y, int(batch))
    if rc:
        raise _lib.QlinError("qlin_conv_silu_update", rc)
    return y
