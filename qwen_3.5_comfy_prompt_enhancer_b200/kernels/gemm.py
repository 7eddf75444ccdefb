"""INT8 GEMM entry points -- drop-in for the reference's ``kernels/gemm.py``.

Same names, signatures, in-place outputs and return values as the reference;
the work runs in the sm_100a kernels of ``libqlin.so`` (``include/qlin.h``).
Tile keyword arguments (``block_m``, ``block_n``, ``group_m``) are accepted for
signature compatibility and ignored: tiles are chosen per launch by the
library.  ``block_k`` must stay 64 (= ``GROUP``).

W4 weights (``torch.uint8`` packed nibbles) are dispatched to ``w4.py`` exactly
as the reference does (kernels/gemm.py:15-17).
"""
import torch

from .. import _lib
from ._host import need_block_k
from .common import GROUP  # noqa: F401  (re-exported like the reference)
from .w4 import gemm_w4, mlp_gate_up_quant_w4, proj3_w4  # noqa: F401  (the W4 names, as the reference exposes them)

_U8 = torch.uint8


def _is_w4(b):
    """W4 checkpoints store uint8 packed nibbles; W8 stores int8 (kernels/gemm.py:15-17)."""
    return b.dtype == _U8


def gemm_i8(a_q, a_s, b, b_s, out, residual=None, block_m=None, block_n=None, block_k=64,
            group_m=8, b_z=None):
    """out[M,N] (bf16) = (a_q * a_s) @ (b * b_s), optional residual add (kernels/gemm.py:60-92).

    ``b`` is int8 [K,N] with one fp32 scale per column, or uint8 [K//2,N]
    packed int4 with per-group scales (then dispatched to ``gemm_w4``).
    ``a_s`` holds one scale per GROUP of K ([M, K//GROUP]).  ``residual`` may
    alias ``out``.  Returns ``out``.
    """
    if block_k != 64:
        need_block_k(block_k)
    if b.dtype == _U8:
        # the W4 entry point, called here directly (one Python frame less per call)
        rc = _lib.ext().gemm_w4(a_q, a_s, b, b_s, out, residual, b_z)
        if rc:
            raise _lib.QlinError("qlin_gemm_w4", rc)
        return out
    rc = _lib.ext().gemm_i8(a_q, a_s, b, b_s, out, residual)
    if rc:
        raise _lib.QlinError("qlin_gemm_i8", rc)
    return out


def mlp_gate_up(a_q, a_s, wg, wsg, wu, wsu, out, block_k=64):
    """h = silu(gate(x)) * up(x) stored bf16 [M,N] (kernels/gemm.py:95-151)."""
    if block_k != 64:
        need_block_k(block_k)
    rc = _lib.ext().mlp_gate_up(a_q, a_s, wg, wsg, wu, wsu, out)
    if rc:
        raise _lib.QlinError("qlin_mlp_gate_up", rc)
    return out


def mlp_gate_up_quant(a_q, a_s, wg, wsg, wu, wsu, out_q, out_s, block_k=64, zg=None, zu=None):
    """Fused gate/up MLP + int8 quantisation of h, the down_proj input
    (kernels/gemm.py:154-231).  Returns ``(out_q, out_s)``."""
    if block_k != 64:
        need_block_k(block_k)
    if wg.dtype == _U8:
        rc = _lib.ext().mlp_gate_up_quant_w4(a_q, a_s, wg, wsg, wu, wsu, out_q, out_s, zg, zu)
        if rc:
            raise _lib.QlinError("qlin_mlp_gate_up_quant_w4", rc)
        return out_q, out_s
    rc = _lib.ext().mlp_gate_up_quant(a_q, a_s, wg, wsg, wu, wsu, out_q, out_s)
    if rc:
        raise _lib.QlinError("qlin_mlp_gate_up_quant", rc)
    return out_q, out_s


def proj3(a_q, a_s, w1, s1, w2, s2, w3, s3, out, block_k=64, z1=None, z2=None, z3=None):
    """Three projections sharing A, written into out[:, 0:N1 | N1:N1+N2 | ...]
    (kernels/gemm.py:234-312).  ``None`` weights contribute no columns."""
    if block_k != 64:
        need_block_k(block_k)
    if w1.dtype == _U8:
        rc = _lib.ext().proj3_w4(a_q, a_s, w1, s1, w2, s2, w3, s3, out, z1, z2, z3)
        if rc:
            raise _lib.QlinError("qlin_proj3_w4", rc)
        return out
    rc = _lib.ext().proj3(a_q, a_s, w1, s1, w2, s2, w3, s3, out)
    if rc:
        raise _lib.QlinError("qlin_proj3", rc)
    return out
