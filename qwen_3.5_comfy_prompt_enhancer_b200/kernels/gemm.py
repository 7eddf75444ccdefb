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

from ._host import call, need, need_block_k, need_rows, ptr, stream_of
from .common import GROUP  # noqa: F401  (re-exported like the reference)
from .w4 import gemm_w4, mlp_gate_up_quant_w4, proj3_w4


def _is_w4(b):
    """W4 checkpoints store uint8 packed nibbles; W8 stores int8 (kernels/gemm.py:15-17)."""
    return b.dtype == torch.uint8


def _acts(a_q, a_s):
    need(a_q, "a_q", torch.int8, 2)
    need(a_s, "a_s", torch.float32, 2)
    M, K = a_q.shape
    if a_s.shape[0] != M or a_s.shape[1] * GROUP != K:
        raise ValueError(f"a_s must be [M, K/64] = [{M}, {K // GROUP}], got {tuple(a_s.shape)}")
    return M, K


def _w8(b, b_s, K, name="b"):
    need(b, name, torch.int8, 2)
    need(b_s, name + "_s", torch.float32, 1)
    if b.shape[0] != K:
        raise ValueError(f"{name} must be [K={K}, N], got {tuple(b.shape)}")
    if b_s.shape[0] != b.shape[1]:
        raise ValueError(f"{name} scales must have N={b.shape[1]} entries, got {b_s.shape[0]}")
    return b.shape[1]


def gemm_i8(a_q, a_s, b, b_s, out, residual=None, block_m=None, block_n=None, block_k=64,
            group_m=8, b_z=None):
    """out[M,N] (bf16) = (a_q * a_s) @ (b * b_s), optional residual add (kernels/gemm.py:60-92).

    ``b`` is int8 [K,N] with one fp32 scale per column, or uint8 [K//2,N]
    packed int4 with per-group scales (then dispatched to ``gemm_w4``).
    ``a_s`` holds one scale per GROUP of K ([M, K//GROUP]).  ``residual`` may
    alias ``out``.  Returns ``out``.
    """
    if _is_w4(b):
        return gemm_w4(a_q, a_s, b, b_s, out, residual=residual, b_z=b_z, block_m=block_m,
                       block_n=block_n, block_k=block_k, group_m=group_m)
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    N = _w8(b, b_s, K)
    need_rows(out, "out", torch.bfloat16)
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out must be [{M}, {N}], got {tuple(out.shape)}")
    if residual is not None:
        need_rows(residual, "residual", torch.bfloat16)
        if tuple(residual.shape) != (M, N):
            raise ValueError(f"residual must be [{M}, {N}], got {tuple(residual.shape)}")
    call("qlin_gemm_i8", a_q.device, ptr(a_q), ptr(a_s), M, K, ptr(b), ptr(b_s), N,
         ptr(out), out.stride(0), ptr(residual),
         residual.stride(0) if residual is not None else 0, stream_of(a_q))
    return out


def mlp_gate_up(a_q, a_s, wg, wsg, wu, wsu, out, block_k=64):
    """h = silu(gate(x)) * up(x) stored bf16 [M,N] (kernels/gemm.py:95-151)."""
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    N = _w8(wg, wsg, K, "wg")
    if _w8(wu, wsu, K, "wu") != N:
        raise ValueError("gate and up weights must have the same N")
    need(out, "out", torch.bfloat16, 2)
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out must be [{M}, {N}], got {tuple(out.shape)}")
    call("qlin_mlp_gate_up", a_q.device, ptr(a_q), ptr(a_s), M, K, ptr(wg), ptr(wsg), ptr(wu),
         ptr(wsu), N, ptr(out), out.stride(0), stream_of(a_q))
    return out


def _quant_out(out_q, out_s, M, N):
    need(out_q, "out_q", torch.int8, 2)
    need(out_s, "out_s", torch.float32, 2)
    if tuple(out_q.shape) != (M, N) or tuple(out_s.shape) != (M, N // GROUP):
        raise ValueError(f"out_q/out_s must be [{M}, {N}] / [{M}, {N // GROUP}]")


def mlp_gate_up_quant(a_q, a_s, wg, wsg, wu, wsu, out_q, out_s, block_k=64, zg=None, zu=None):
    """Fused gate/up MLP + int8 quantisation of h, the down_proj input
    (kernels/gemm.py:154-231).  Returns ``(out_q, out_s)``."""
    if _is_w4(wg):
        return mlp_gate_up_quant_w4(a_q, a_s, wg, wsg, wu, wsu, out_q, out_s, zg=zg, zu=zu,
                                    block_k=block_k)
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    N = _w8(wg, wsg, K, "wg")
    if _w8(wu, wsu, K, "wu") != N:
        raise ValueError("gate and up weights must have the same N")
    _quant_out(out_q, out_s, M, N)
    call("qlin_mlp_gate_up_quant", a_q.device, ptr(a_q), ptr(a_s), M, K, ptr(wg), ptr(wsg),
         ptr(wu), ptr(wsu), N, ptr(out_q), ptr(out_s), stream_of(a_q))
    return out_q, out_s


def proj3(a_q, a_s, w1, s1, w2, s2, w3, s3, out, block_k=64, z1=None, z2=None, z3=None):
    """Three projections sharing A, written into out[:, 0:N1 | N1:N1+N2 | ...]
    (kernels/gemm.py:234-312).  ``None`` weights contribute no columns."""
    if _is_w4(w1):
        return proj3_w4(a_q, a_s, w1, s1, w2, s2, w3, s3, out, block_k=block_k, z1=z1, z2=z2,
                        z3=z3)
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    segs = []
    for i, (w, s) in enumerate(((w1, s1), (w2, s2), (w3, s3))):
        if w is None:
            segs += [None, None, 0]
        else:
            segs += [ptr(w), ptr(s), _w8(w, s, K, f"w{i + 1}")]
    NT = segs[2] + segs[5] + segs[8]
    need_rows(out, "out", torch.bfloat16)
    if out.shape[0] != M or out.shape[1] < NT:
        raise ValueError(f"out must be [{M}, >={NT}], got {tuple(out.shape)}")
    call("qlin_proj3", a_q.device, ptr(a_q), ptr(a_s), M, K, *segs, ptr(out), out.stride(0),
         stream_of(a_q))
    return out
