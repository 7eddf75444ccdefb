"""W4 GEMM entry points -- drop-in for the reference's ``kernels/w4.py``.

Engine W4 layout (kernels/w4.py:3-15): ``W`` uint8 [K//2, N] (even K in the
low nibble, odd K in the high nibble), ``WS`` bf16 [K//WGRP, N] group scales,
optional ``Z`` uint8 [K//WGRP, N] per-group zeros; a stored element decodes to
``nibble - z`` (z = 8 without zeros).  WGRP = K // WS.shape[0] must be 32 or a
multiple of 64.  Tile keyword arguments are accepted and ignored.
"""
import torch

from ._host import call, need, need_block_k, need_rows, ptr, stream_of
from .common import GROUP


def _acts(a_q, a_s):
    need(a_q, "a_q", torch.int8, 2)
    need(a_s, "a_s", torch.float32, 2)
    M, K = a_q.shape
    if a_s.shape[0] != M or a_s.shape[1] * GROUP != K:
        raise ValueError(f"a_s must be [M, K/64] = [{M}, {K // GROUP}], got {tuple(a_s.shape)}")
    return M, K


def _w4(b, b_s, b_z, K, name="b"):
    """Validate one W4 weight; returns (N, WGRP)."""
    need(b, name, torch.uint8, 2)
    need(b_s, name + "_s", torch.bfloat16, 2)
    if b.shape[0] * 2 != K:
        raise ValueError(f"{name} must be [K//2={K // 2}, N], got {tuple(b.shape)}")
    N = b.shape[1]
    if b_s.shape[1] != N or b_s.shape[0] == 0 or K % b_s.shape[0] != 0:
        raise ValueError(f"{name} scales must be [K//WGRP, {N}], got {tuple(b_s.shape)}")
    wgrp = K // b_s.shape[0]
    if b_z is not None:
        need(b_z, name + "_z", torch.uint8, 2)
        if tuple(b_z.shape) != tuple(b_s.shape):
            raise ValueError(f"{name} zeros must match scales {tuple(b_s.shape)}, got {tuple(b_z.shape)}")
    return N, wgrp


def gemm_w4(a_q, a_s, b, b_s, out, residual=None, b_z=None, block_m=None, block_n=None, block_k=64,
            group_m=8, num_warps=None, num_stages=3):
    """out[M,N] (bf16) = (a_q * a_s) @ unpack(b) * b_s, optional residual add
    (kernels/w4.py:139-166).  Returns ``out``."""
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    N, wgrp = _w4(b, b_s, b_z, K)
    need_rows(out, "out", torch.bfloat16)
    if tuple(out.shape) != (M, N):
        raise ValueError(f"out must be [{M}, {N}], got {tuple(out.shape)}")
    if residual is not None:
        need_rows(residual, "residual", torch.bfloat16)
        if tuple(residual.shape) != (M, N):
            raise ValueError(f"residual must be [{M}, {N}], got {tuple(residual.shape)}")
    call("qlin_gemm_w4", a_q.device, ptr(a_q), ptr(a_s), M, K, ptr(b), ptr(b_s), ptr(b_z), N, wgrp,
         ptr(out), out.stride(0), ptr(residual),
         residual.stride(0) if residual is not None else 0, stream_of(a_q))
    return out


def proj3_w4(a_q, a_s, w1, s1, w2, s2, w3, s3, out, z1=None, z2=None, z3=None, block_k=64):
    """Three W4 projections sharing one activation (kernels/w4.py:220-251).

    A segment whose zeros are ``None`` decodes with zero = 8.  (The reference
    instead borrows another segment's zero tensor when only some segments have
    zeros, kernels/w4.py:238-241; engine checkpoints never mix the two.)
    """
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    segs = []
    wgrp = None
    for i, (w, s, z) in enumerate(((w1, s1, z1), (w2, s2, z2), (w3, s3, z3))):
        if w is None:
            segs += [None, None, None, 0]
            continue
        n, wg = _w4(w, s, z, K, f"w{i + 1}")
        if wgrp is None:
            wgrp = wg
        elif wg != wgrp:
            raise ValueError("all proj3_w4 segments must share one weight group size")
        segs += [ptr(w), ptr(s), ptr(z), n]
    NT = segs[3] + segs[7] + segs[11]
    need_rows(out, "out", torch.bfloat16)
    if out.shape[0] != M or out.shape[1] < NT:
        raise ValueError(f"out must be [{M}, >={NT}], got {tuple(out.shape)}")
    call("qlin_proj3_w4", a_q.device, ptr(a_q), ptr(a_s), M, K, *segs, wgrp or 64, ptr(out),
         out.stride(0), stream_of(a_q))
    return out


def mlp_gate_up_quant_w4(a_q, a_s, wg, sg, wu, su, out_q, out_s, zg=None, zu=None, block_k=64):
    """W4 gate/up fusion + int8 quantisation of h (kernels/w4.py:300-323).
    Returns ``(out_q, out_s)``."""
    need_block_k(block_k)
    M, K = _acts(a_q, a_s)
    N, wgrp = _w4(wg, sg, zg, K, "wg")
    Nu, wgrp_u = _w4(wu, su, zu, K, "wu")
    if Nu != N or wgrp_u != wgrp:
        raise ValueError("gate and up weights must have the same N and group size")
    need(out_q, "out_q", torch.int8, 2)
    need(out_s, "out_s", torch.float32, 2)
    if tuple(out_q.shape) != (M, N) or tuple(out_s.shape) != (M, N // GROUP):
        raise ValueError(f"out_q/out_s must be [{M}, {N}] / [{M}, {N // GROUP}]")
    call("qlin_mlp_gate_up_quant_w4", a_q.device, ptr(a_q), ptr(a_s), M, K, ptr(wg), ptr(sg),
         ptr(zg), ptr(wu), ptr(su), ptr(zu), N, wgrp, ptr(out_q), ptr(out_s), stream_of(a_q))
    return out_q, out_s
