"""W4 GEMM entry points -- drop-in for the reference's ``kernels/w4.py``.

Engine W4 layout (kernels/w4.py:3-15): ``W`` uint8 [K//2, N] (even K in the
low nibble, odd K in the high nibble), ``WS`` bf16 [K//WGRP, N] group scales,
optional ``Z`` uint8 [K//WGRP, N] per-group zeros; a stored element decodes to
``nibble - z`` (z = 8 without zeros).  WGRP = K // WS.shape[0] must be 32 or a
multiple of 64.  Tile keyword arguments are accepted and ignored.
"""
from .. import _lib
from ._host import need_block_k


def gemm_w4(a_q, a_s, b, b_s, out, residual=None, b_z=None, block_m=None, block_n=None, block_k=64,
            group_m=8, num_warps=None, num_stages=3):
    """out[M,N] (bf16) = (a_q * a_s) @ unpack(b) * b_s, optional residual add
    (kernels/w4.py:139-166).  Returns ``out``."""
    if block_k != 64:
        need_block_k(block_k)
    rc = _lib.ext().gemm_w4(a_q, a_s, b, b_s, out, residual, b_z)
    if rc:
        raise _lib.QlinError("qlin_gemm_w4", rc)
    return out


def proj3_w4(a_q, a_s, w1, s1, w2, s2, w3, s3, out, z1=None, z2=None, z3=None, block_k=64):
    """Three W4 projections sharing one activation (kernels/w4.py:220-251).

    A segment whose zeros are ``None`` decodes with zero = 8.  (The reference
    instead borrows another segment's zero tensor when only some segments have
    zeros, kernels/w4.py:238-241; engine checkpoints never mix the two.)
    All segments must share one weight group size.
    """
    if block_k != 64:
        need_block_k(block_k)
    rc = _lib.ext().proj3_w4(a_q, a_s, w1, s1, w2, s2, w3, s3, out, z1, z2, z3)
    if rc:
        raise _lib.QlinError("qlin_proj3_w4", rc)
    return out


def mlp_gate_up_quant_w4(a_q, a_s, wg, sg, wu, su, out_q, out_s, zg=None, zu=None, block_k=64):
    """W4 gate/up fusion + int8 quantisation of h (kernels/w4.py:300-323).
    Returns ``(out_q, out_s)``."""
    if block_k != 64:
        need_block_k(block_k)
    rc = _lib.ext().mlp_gate_up_quant_w4(a_q, a_s, wg, sg, wu, su, out_q, out_s, zg, zu)
    if rc:
        raise _lib.QlinError("qlin_mlp_gate_up_quant_w4", rc)
    return out_q, out_s
