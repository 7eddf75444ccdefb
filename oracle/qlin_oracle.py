"""CPU oracle for the quantised-linear hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The shipped package calls CUDA through the C-ABI
library and has no CPU path.

Every function restates, in numpy, the arithmetic of one reference function of
``kernels/gemm.py``, ``kernels/w4.py``, ``kernels/norm.py`` (the activation
producers included) or ``kernels/common.py`` (paths relative to the reference project root; line
numbers cited per function).  The restatement is exact at the level the
reference defines it:

* integer parts bit-exact: int32 sums per 64-element K block (per ``SUB``
  sub-block for W4), nibble decode ``nibble - z``, int8 activation codes;
* fp32 epilogue in the reference's program order, one rounding per numpy
  float32 operation (no fused multiply-add), K blocks summed in ascending
  order;
* bf16 output rounding selectable: ``"rne"`` (round-to-nearest-even, what a
  GPU build of the reference does) or ``"trunc"`` (what Triton's CPU
  interpreter does; used only to pin this oracle against fixtures produced by
  running the reference under ``TRITON_INTERPRET=1``, see
  ``tests/golden/make_golden.py``).

The oracle is pinned bit-exactly against those fixtures by
``tests/test_oracle_golden.py``.

``dequant_matmul_*`` are the reference's own pure-PyTorch CPU formulation
(``.dev/test_kernels.py:40-41``) used as the timed CPU baseline.
"""
from __future__ import annotations

import numpy as np

GROUP = 64  # kernels/common.py:7


# ----------------------------------------------------------------------------
# bf16 helpers (bf16 is stored as uint16 bit patterns in numpy)
# ----------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray, mode: str = "rne") -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16).  ``mode`` is "rne" or "trunc"."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    if mode == "trunc":
        r = b >> 16
    elif mode == "rne":
        r = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
        nan = np.isnan(x)
        r = np.where(nan, (b >> 16) | 0x40, r)
    else:
        raise ValueError(mode)
    return r.astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray, mode: str = "rne") -> np.ndarray:
    """x.to(bf16).to(fp32) as the reference writes it (gemm.py:200, w4.py:286)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x, mode))


# ----------------------------------------------------------------------------
# common.py helpers
# ----------------------------------------------------------------------------

def round_i8(v: np.ndarray) -> np.ndarray:
    """kernels/common.py:24-29: trunc(v + (v >= 0 ? 0.5 : -0.5)) clamped to +-127.

    The +-0.5 add is an fp32 operation (it can itself round), the conversion
    truncates toward zero.  This is round-half-away-from-zero, not numpy's
    half-to-even ``np.round``.
    """
    v = np.asarray(v, dtype=np.float32)
    half = np.where(v >= np.float32(0.0), np.float32(0.5), np.float32(-0.5)).astype(np.float32)
    t = (v + half).astype(np.float32)
    with np.errstate(invalid="ignore"):
        r = np.trunc(t)
    r = np.clip(r, -127, 127)
    return r.astype(np.int8)


def silu(x: np.ndarray) -> np.ndarray:
    """kernels/common.py:32-34 with Triton's ``sigmoid = 1 / (1 + exp(-x))``."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        e = np.exp(-x).astype(np.float32)
    sig = (np.float32(1.0) / (np.float32(1.0) + e).astype(np.float32)).astype(np.float32)
    return (x * sig).astype(np.float32)


def quant_groups(y: np.ndarray):
    """kernels/norm.py:15-25 (``_quant_groups``): per row, per 64-group.

    ``s = max(amax / 127, 1e-8)`` (IEEE fp32 division), ``q = round_i8(y / s)``
    (true division, not multiply by reciprocal).  Returns (int8 [M,K],
    fp32 [M,K/64]).
    """
    y = np.asarray(y, dtype=np.float32)
    M, K = y.shape
    assert K % GROUP == 0
    y3 = y.reshape(M, K // GROUP, GROUP)
    amax = np.abs(y3).max(axis=2).astype(np.float32)
    s = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-8)).astype(np.float32)
    q = round_i8((y3 / s[:, :, None]).astype(np.float32))
    return q.reshape(M, K), s


def quant_row(x_bits: np.ndarray):
    """kernels/norm.py:75-92: bf16 X [M,K] -> (int8 [M,K], fp32 [M,K/64])."""
    return quant_groups(bf16_bits_to_f32(x_bits))


# ----------------------------------------------------------------------------
# int8 x int8 -> int32 block sums
# ----------------------------------------------------------------------------

def _block_sum(a_q: np.ndarray, w: np.ndarray, k0: int, blk: int) -> np.ndarray:
    """int32 [M, N]: exact sum over K block [k0, k0+blk) of a[m,k] * w[k,n].

    Computed in float64 (BLAS): every partial sum of int8 x int8 products over
    a block of <= 64 is an integer below 2^21, exactly representable."""
    a = a_q[:, k0:k0 + blk].astype(np.float64)
    ww = w[k0:k0 + blk].astype(np.float64)
    return (a @ ww).astype(np.int32)


def _block_sums(a_q: np.ndarray, w: np.ndarray, blk: int) -> np.ndarray:
    """int32 [K/blk, M, N]: exact sum over each K block of a[m,k] * w[k,n]."""
    M, K = a_q.shape
    assert w.shape[0] == K and K % blk == 0
    return np.stack([_block_sum(a_q, w, k0, blk) for k0 in range(0, K, blk)])


def unpack_w4(b: np.ndarray, b_z, wgrp: int) -> np.ndarray:
    """kernels/w4.py:3-15, 48-61, 78-88: packed uint8 [K/2, N] -> int8 [K, N].

    Byte j of column n holds k = 2j in the low nibble and k = 2j+1 in the high
    nibble; the signed value is ``nibble - z`` with ``z`` the per-(group, n)
    zero (uint8 [K/WG, N]) or 8 when there is none.
    """
    b = np.asarray(b, dtype=np.uint8)
    K2, N = b.shape
    K = 2 * K2
    nib = np.empty((K, N), dtype=np.int32)
    nib[0::2] = b & 0x0F
    nib[1::2] = (b >> 4) & 0x0F
    if b_z is None:
        z = np.full((K, N), 8, dtype=np.int32)
    else:
        z = np.repeat(np.asarray(b_z, dtype=np.int32), wgrp, axis=0)
    return (nib - z).astype(np.int8)


# ----------------------------------------------------------------------------
# a1: gemm_i8  (kernels/gemm.py:20-92)
# ----------------------------------------------------------------------------

def gemm_i8_f32(a_q, a_s, b, b_s, residual_f32=None) -> np.ndarray:
    """fp32 result of gemm_i8 before the bf16 store (gemm.py:38-55).

    ``out += float(int32 block dot) * a_s[m, kb]`` for kb ascending, then
    ``out *= b_s[n]``, then ``out += residual``.
    """
    a_s = np.asarray(a_s, dtype=np.float32)
    b_s = np.asarray(b_s, dtype=np.float32)
    M, K = a_q.shape
    N = b.shape[1]
    out = np.zeros((M, N), dtype=np.float32)
    for kb in range(K // GROUP):
        blk = _block_sum(a_q, b, kb * GROUP, GROUP)
        prod = (blk.astype(np.float32) * a_s[:, kb:kb + 1]).astype(np.float32)
        out = (out + prod).astype(np.float32)
    out = (out * b_s[None, :]).astype(np.float32)
    if residual_f32 is not None:
        out = (out + residual_f32).astype(np.float32)
    return out


def gemm_i8(a_q, a_s, b, b_s, residual_bits=None, mode="rne") -> np.ndarray:
    """kernels/gemm.py:60-92 -> bf16 bits [M,N]."""
    res = None if residual_bits is None else bf16_bits_to_f32(residual_bits)
    return f32_to_bf16_bits(gemm_i8_f32(a_q, a_s, b, b_s, res), mode)


# ----------------------------------------------------------------------------
# a5: gemm_w4  (kernels/w4.py:64-166)
# ----------------------------------------------------------------------------

def w4_sub(wgrp: int) -> int:
    """w4.py:113: SUB = BLOCK_K if WGRP >= BLOCK_K else WGRP."""
    return GROUP if wgrp >= GROUP else wgrp


def gemm_w4_f32(a_q, a_s, b, b_s_bits, b_z=None, residual_f32=None) -> np.ndarray:
    """fp32 result of gemm_w4 before the bf16 store (w4.py:124-134).

    Per sub-block of ``SUB = min(WGRP, 64)`` at k0 (ascending):
    ``out += float(int32 dot) * (a_s[m, k0/64] * float(ws[k0/WGRP, n]))``.
    """
    a_s = np.asarray(a_s, dtype=np.float32)
    M, K = a_q.shape
    ws = bf16_bits_to_f32(b_s_bits)
    wgrp = K // ws.shape[0]
    sub = w4_sub(wgrp)
    w = unpack_w4(b, b_z, wgrp)
    sums = _block_sums(a_q, w, sub)
    N = w.shape[1]
    out = np.zeros((M, N), dtype=np.float32)
    for i in range(K // sub):
        k0 = i * sub
        sc = (a_s[:, k0 // GROUP][:, None] * ws[k0 // wgrp][None, :]).astype(np.float32)
        prod = (sums[i].astype(np.float32) * sc).astype(np.float32)
        out = (out + prod).astype(np.float32)
    if residual_f32 is not None:
        out = (out + residual_f32).astype(np.float32)
    return out


def gemm_w4(a_q, a_s, b, b_s_bits, b_z=None, residual_bits=None, mode="rne"):
    """kernels/w4.py:139-166 -> bf16 bits [M,N]."""
    res = None if residual_bits is None else bf16_bits_to_f32(residual_bits)
    return f32_to_bf16_bits(gemm_w4_f32(a_q, a_s, b, b_s_bits, b_z, res), mode)


# ----------------------------------------------------------------------------
# a2 / a6: proj3  (kernels/gemm.py:234-312, kernels/w4.py:169-251)
# ----------------------------------------------------------------------------

def proj3(a_q, a_s, segs, mode="rne"):
    """Three projections sharing A, written side by side (gemm.py:252-287).

    ``segs`` is a list of ``(w, s, z)``; ``w`` int8 [K,N_i] (W8, ``s`` fp32
    [N_i]) or uint8 [K/2,N_i] (W4, ``s`` bf16 bits [K/WG,N_i], ``z`` optional
    zeros).  ``None`` entries are skipped (N_i = 0).  Returns bf16 bits
    [M, sum N_i].
    """
    parts = []
    for seg in segs:
        if seg is None or seg[0] is None:
            continue
        w, s, z = seg
        if w.dtype == np.uint8:
            parts.append(gemm_w4(a_q, a_s, w, s, z, None, mode))
        else:
            parts.append(gemm_i8(a_q, a_s, w, s, None, mode))
    return np.concatenate(parts, axis=1)


# ----------------------------------------------------------------------------
# a3 / a4 / a7: fused gate/up
# ----------------------------------------------------------------------------

def _gate_up_w8_h(a_q, a_s, wg, sg, wu, su):
    """gemm.py:180-197: h = silu(g * sg) * (u * su), fp32."""
    g = gemm_i8_f32(a_q, a_s, wg, np.ones_like(np.asarray(sg, dtype=np.float32)))
    u = gemm_i8_f32(a_q, a_s, wu, np.ones_like(np.asarray(su, dtype=np.float32)))
    # gemm_i8_f32 multiplies by 1.0 (exact); apply the real scales here in the
    # reference order: silu(g * sg) * (u * su).
    g = (g * np.asarray(sg, dtype=np.float32)[None, :]).astype(np.float32)
    u = (u * np.asarray(su, dtype=np.float32)[None, :]).astype(np.float32)
    return (silu(g) * u).astype(np.float32)


def mlp_gate_up(a_q, a_s, wg, sg, wu, su, mode="rne"):
    """kernels/gemm.py:95-151 -> bf16 bits [M,N]."""
    return f32_to_bf16_bits(_gate_up_w8_h(a_q, a_s, wg, sg, wu, su), mode)


def _quant_h(h, mode):
    """gemm.py:198-211 / w4.py:285-297: round h through bf16, then per-64 quant."""
    return quant_groups(bf16_round(h, mode))


def mlp_gate_up_quant(a_q, a_s, wg, sg, wu, su, mode="rne"):
    """kernels/gemm.py:154-231 -> (int8 [M,N], fp32 [M,N/64])."""
    return _quant_h(_gate_up_w8_h(a_q, a_s, wg, sg, wu, su), mode)


def mlp_gate_up_quant_w4(a_q, a_s, wg, sg_bits, wu, su_bits, zg=None, zu=None, mode="rne"):
    """kernels/w4.py:254-323: g, u with scales inside the K loop, h = silu(g)*u."""
    g = gemm_w4_f32(a_q, a_s, wg, sg_bits, zg)
    u = gemm_w4_f32(a_q, a_s, wu, su_bits, zu)
    h = (silu(g) * u).astype(np.float32)
    return _quant_h(h, mode)


# ----------------------------------------------------------------------------
# f1: activation producers  (kernels/norm.py)
# ----------------------------------------------------------------------------
# The reference reduces with ``tl.sum`` over a row padded with zeros to a
# power-of-two block; the restatement sums the same padded float32 array with
# numpy (the CPU interpreter's own reduction), so the golden fixtures pin it
# bit for bit.  A GPU build sums in another order: its results agree to a
# few fp32 ulps, and the tests say how that reaches the int8 codes.

def _next_pow2(n: int) -> int:
    return 1 << max(0, n - 1).bit_length()


def _pad(x: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(x.shape[:-1] + (n,), dtype=np.float32)
    out[..., :x.shape[-1]] = x
    return out


def _rsqrt(v):
    """tl.rsqrt: 1 / sqrt(v) in float32 (correctly rounded sqrt, then division)."""
    v = np.asarray(v, dtype=np.float32)
    return (np.float32(1.0) / np.sqrt(v)).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    """triton.language.standard.sigmoid: 1 / (1 + exp(-x)) in float32."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore"):
        e = np.exp(-x).astype(np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + e).astype(np.float32)).astype(np.float32)


def softplus(x: np.ndarray) -> np.ndarray:
    """kernels/common.py:37-39: x > 20 ? x : log(1 + exp(min(x, 20)))."""
    x = np.asarray(x, dtype=np.float32)
    e = np.exp(np.minimum(x, np.float32(20.0))).astype(np.float32)
    lg = np.log((np.float32(1.0) + e).astype(np.float32)).astype(np.float32)
    return np.where(x > np.float32(20.0), x, lg).astype(np.float32)


def rmsnorm_y(x_bits, w_bits, eps=1e-6, one_plus=True) -> np.ndarray:
    """kernels/norm.py:31-41: the fp32 rows ``x * rsqrt(var + eps) * w`` that
    rmsnorm_quant quantises; var = sum(x*x) / K over the row padded to
    BLOCK_K = max(256, next_pow2(K))."""
    x = bf16_bits_to_f32(x_bits)
    M, K = x.shape
    blk = max(256, _next_pow2(K))
    xp = _pad(x, blk)
    w = _pad(bf16_bits_to_f32(w_bits)[None, :], blk)[0]
    if one_plus:
        w = (w + np.float32(1.0)).astype(np.float32)
    out = np.empty((M, K), dtype=np.float32)
    for m in range(M):
        ss = np.sum((xp[m] * xp[m]).astype(np.float32), dtype=np.float32)
        var = (np.float32(ss) / np.float32(K)).astype(np.float32)
        r = _rsqrt((var + np.float32(eps)).astype(np.float32))
        out[m] = ((xp[m] * r).astype(np.float32) * w).astype(np.float32)[:K]
    return out


def rmsnorm_quant(x_bits, w_bits, eps=1e-6, one_plus=True):
    """kernels/norm.py:28-57 -> (int8 [M,K], fp32 [M,K/64])."""
    return quant_groups(rmsnorm_y(x_bits, w_bits, eps, one_plus))


def norm_gated_y(v_bits, z_bits, w_bits, eps=1e-6) -> np.ndarray:
    """kernels/norm.py:111-123 / 150-164: per (token, head) of HD dims,
    ``x * rsqrt(sum(x*x)/HD + eps) * w * silu(z)`` in fp32 (before any bf16
    rounding); the head is padded to BLOCK = max(128, next_pow2(HD))."""
    v = bf16_bits_to_f32(v_bits)
    T, N = v.shape
    z = bf16_bits_to_f32(z_bits)[:, :N]
    w = bf16_bits_to_f32(w_bits)
    HD = w.shape[0]
    NV = N // HD
    blk = max(128, _next_pow2(HD))
    out = np.empty((T, N), dtype=np.float32)
    for t in range(T):
        for h in range(NV):
            x = _pad(v[t, h * HD:(h + 1) * HD][None, :], blk)[0]
            ss = np.sum((x * x).astype(np.float32), dtype=np.float32)
            var = (np.float32(ss) / np.float32(HD)).astype(np.float32)
            r = _rsqrt((var + np.float32(eps)).astype(np.float32))
            xx = x[:HD]
            y = ((xx * r).astype(np.float32) * w).astype(np.float32)
            out[t, h * HD:(h + 1) * HD] = (y * silu(z[t, h * HD:(h + 1) * HD])).astype(np.float32)
    return out


def norm_gated_quant(v_bits, z_bits, w_bits, eps=1e-6, mode="rne"):
    """kernels/norm.py:95-137: y rounded through bf16, then per-64 quantisation
    (groups never straddle heads: HD is a multiple of 64)."""
    return quant_groups(bf16_round(norm_gated_y(v_bits, z_bits, w_bits, eps), mode))


def norm_gated(v_bits, z_bits, w_bits, eps=1e-6, mode="rne"):
    """kernels/norm.py:141-165 -> bf16 bits [T, N]."""
    return f32_to_bf16_bits(norm_gated_y(v_bits, z_bits, w_bits, eps), mode)


def gate_mul_y(a_bits, g_bits, hd=256) -> np.ndarray:
    """kernels/norm.py:175-181: a * sigmoid(gate), gate of column n at column
    (n // hd) * 2 hd + hd + n % hd of the g row."""
    a = bf16_bits_to_f32(a_bits)
    M, N = a.shape
    g = bf16_bits_to_f32(g_bits)
    n = np.arange(N)
    gcol = (n // hd) * (2 * hd) + hd + (n % hd)
    return (a * sigmoid(g[:, gcol])).astype(np.float32)


def gate_mul_quant(a_bits, g_bits, hd=256):
    """kernels/norm.py:168-188 -> (int8 [M,N], fp32 [M,N/64])."""
    return quant_groups(gate_mul_y(a_bits, g_bits, hd))


def silu_mul_quant(g_bits, u_bits):
    """kernels/norm.py:191-208: silu(g) * u quantised per 64."""
    g = bf16_bits_to_f32(g_bits)
    u = bf16_bits_to_f32(u_bits)
    return quant_groups((silu(g) * u).astype(np.float32))


def gate_proj(a_q, a_s, wb_bits, wa_bits, dt_bits, alog_bits):
    """kernels/norm.py:211-240 -> (beta fp32 [M,NB], gate fp32 [M,NB]).

    x = a_q * a_s[k // 64]; b = sum_k wb[n,k] * x[k], av likewise (row padded
    to BLOCK_K = max(256, next_pow2(K))); beta = sigmoid(b);
    gate = -exp(A_log) * softplus(av + dt_bias)."""
    a_q = np.asarray(a_q, dtype=np.int8)
    a_s = np.asarray(a_s, dtype=np.float32)
    M, K = a_q.shape
    blk = max(256, _next_pow2(K))
    wb = _pad(bf16_bits_to_f32(wb_bits), blk)
    wa = _pad(bf16_bits_to_f32(wa_bits), blk)
    dtb = bf16_bits_to_f32(dt_bits)
    alog = bf16_bits_to_f32(alog_bits)
    NB = wb.shape[0]
    beta = np.empty((M, NB), dtype=np.float32)
    gate = np.empty((M, NB), dtype=np.float32)
    for m in range(M):
        x = (a_q[m].astype(np.float32) * np.repeat(a_s[m], GROUP)).astype(np.float32)
        x = _pad(x[None, :], blk)[0]
        b = np.sum((wb * x[None, :]).astype(np.float32), axis=1, dtype=np.float32)
        av = np.sum((wa * x[None, :]).astype(np.float32), axis=1, dtype=np.float32)
        beta[m] = sigmoid(b)
        ea = np.exp(alog).astype(np.float32)
        gate[m] = ((-ea).astype(np.float32) * softplus((av + dtb).astype(np.float32))).astype(np.float32)
    return beta, gate


# ----------------------------------------------------------------------------
# f2: decode-step neighbours  (kernels/attention.py, kernels/linear_attn.py)
# ----------------------------------------------------------------------------

def _norm_rope(x, w, pos, invf, rd, eps, scale):
    """attention.py:20-67 (_norm_rope_store) before the store, fp32: RMSNorm
    with (1 + w) over HD, then rotate-half RoPE on the first rd dims, times
    `scale`.  Returns (plo, phi, yr*scale) as one HD vector."""
    HD = x.shape[0]
    d2 = rd // 2
    blk = HD  # the reference loads the tail with arange(HD) masked to HD - rd
    xlo, xhi = x[:d2], x[d2:rd]
    xr = np.zeros(blk, dtype=np.float32)
    xr[:HD - rd] = x[rd:]
    wlo = (w[:d2] + np.float32(1.0)).astype(np.float32)
    whi = (w[d2:rd] + np.float32(1.0)).astype(np.float32)
    wr = np.zeros(blk, dtype=np.float32)
    wr[:HD - rd] = w[rd:]
    wr = (wr + np.float32(1.0)).astype(np.float32)
    ss = (np.float32(np.sum((xlo * xlo).astype(np.float32), dtype=np.float32))
          + np.float32(np.sum((xhi * xhi).astype(np.float32), dtype=np.float32)))
    ss = (np.float32(ss) + np.float32(np.sum((xr * xr).astype(np.float32), dtype=np.float32))).astype(np.float32)
    var = (np.float32(ss) / np.float32(HD)).astype(np.float32)
    rstd = _rsqrt((var + np.float32(eps)).astype(np.float32))
    ylo = ((xlo * rstd).astype(np.float32) * wlo).astype(np.float32)
    yhi = ((xhi * rstd).astype(np.float32) * whi).astype(np.float32)
    yr = ((xr * rstd).astype(np.float32) * wr).astype(np.float32)[:HD - rd]
    theta = (np.float32(pos) * invf).astype(np.float32)
    c, s = np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)
    sc = np.float32(scale)
    plo = (((ylo * c).astype(np.float32) - (yhi * s).astype(np.float32)).astype(np.float32) * sc).astype(np.float32)
    phi = (((yhi * c).astype(np.float32) + (ylo * s).astype(np.float32)).astype(np.float32) * sc).astype(np.float32)
    return np.concatenate([plo, phi, (yr * sc).astype(np.float32)])


def _quant_vec(y):
    """attention.py:55-60: one amax/127 scale per vector, round_i8 codes."""
    amax = np.float32(np.max(np.abs(y)))
    sc = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-8)).astype(np.float32)
    return round_i8((y / sc).astype(np.float32)), np.float32(sc)


def qk_norm_rope(proj_bits, qn_bits, kn_bits, invf, nq, nkv, hd, pos0, kvc, kvs=None, eps=1e-6,
                 batch=False, mode="rne"):
    """attention.py:70-133.  proj [T, >= (2 nq + 2 nkv) hd] bf16 bits (per q
    head: hd query dims then hd gate dims; then k heads, then v heads).
    Returns q bf16 bits [T, nq*hd] and writes K/V rows into ``kvc`` (a numpy
    array [rows, 2*nkv*hd]: bf16 bits, or int8 with ``kvs`` [rows, 2*nkv]
    fp32).  Row of token t: position pos0 + t; in batch mode row t is
    candidate t at position pos0, in its own slice of kvc.shape[0] // T rows."""
    p = bf16_bits_to_f32(proj_bits)
    T = p.shape[0]
    qn = bf16_bits_to_f32(qn_bits)
    kn = bf16_bits_to_f32(kn_bits)
    invf = np.asarray(invf, dtype=np.float32)
    rd = 2 * invf.shape[0]
    qscale = np.float32(1.0) / np.sqrt(np.float32(hd))
    q = np.empty((T, nq * hd), dtype=np.uint16)
    seq = kvc.shape[0] // T if batch else 0
    int8 = kvs is not None
    for t in range(T):
        pos = pos0 if batch else pos0 + t
        base = t * seq if batch else 0
        for h in range(nq):
            y = _norm_rope(p[t, h * 2 * hd:h * 2 * hd + hd], qn, pos, invf, rd, eps, qscale)
            q[t, h * hd:(h + 1) * hd] = f32_to_bf16_bits(y, mode)
        for j in range(nkv):
            off = 2 * nq * hd
            y = _norm_rope(p[t, off + j * hd:off + (j + 1) * hd], kn, pos, invf, rd, eps, 1.0)
            v = p[t, off + nkv * hd + j * hd:off + nkv * hd + (j + 1) * hd]
            if int8:
                kvc[base + pos, j * hd:(j + 1) * hd], kvs[base + pos, j] = _quant_vec(y)
                kvc[base + pos, (nkv + j) * hd:(nkv + j + 1) * hd], kvs[base + pos, nkv + j] = _quant_vec(v)
            else:
                kvc[base + pos, j * hd:(j + 1) * hd] = f32_to_bf16_bits(y, mode)
                kvc[base + pos, (nkv + j) * hd:(nkv + j + 1) * hd] = f32_to_bf16_bits(v, mode)
    return q


def _kv_rows(kvc, kvs, rows, side, kvh, nkv, hd):
    """fp32 K (side 0) or V (side 1) vectors of one kv head for `rows`."""
    col = (side * nkv + kvh) * hd
    if kvs is None:
        return bf16_bits_to_f32(kvc[rows, col:col + hd])
    return (kvc[rows, col:col + hd].astype(np.float32) * kvs[rows, side * nkv + kvh][:, None]).astype(np.float32)


def attn_decode_f32(q_bits, kvc, pos, kvs=None, batch=1, nq=8, nkv=2, hd=256, block_n=32):
    """attention.py:209-267 before the bf16 store: per candidate b and q head,
    online softmax over positions 0..pos in blocks of block_n (m, l, acc
    rescaled per block, exp in fp32).  q [batch, nq*hd] bf16 bits; kvc rows
    of candidate b are kvc[b*S : (b+1)*S] with S = rows // batch."""
    q = bf16_bits_to_f32(q_bits).reshape(batch, nq, hd)
    S = kvc.shape[0] // batch
    out = np.empty((batch, nq, hd), dtype=np.float32)
    n = pos + 1
    for b in range(batch):
        for h in range(nq):
            kvh = h // (nq // nkv)
            m_i, l_i = np.float32(-np.inf), np.float32(0.0)
            acc = np.zeros(hd, dtype=np.float32)
            for s0 in range(0, n, block_n):
                rows = np.arange(s0, min(n, s0 + block_n))
                k = _kv_rows(kvc, kvs, b * S + rows, 0, kvh, nkv, hd)
                v = _kv_rows(kvc, kvs, b * S + rows, 1, kvh, nkv, hd)
                sc = np.sum((q[b, h][None, :] * k).astype(np.float32), axis=1, dtype=np.float32)
                m_new = np.float32(max(m_i, np.float32(sc.max())))
                p = np.exp((sc - m_new).astype(np.float32)).astype(np.float32)
                alpha = np.float32(np.exp(np.float32(m_i - m_new)))
                l_i = np.float32(np.float32(l_i * alpha) + np.float32(np.sum(p, dtype=np.float32)))
                acc = (acc * alpha).astype(np.float32)
                acc = (acc + np.sum((p[:, None] * v).astype(np.float32), axis=0, dtype=np.float32)).astype(np.float32)
                m_i = m_new
            out[b, h] = (acc / l_i).astype(np.float32)
    return out.reshape(batch, nq * hd)


def attn_decode(q_bits, kvc, pos, kvs=None, batch=1, nq=8, nkv=2, hd=256, mode="rne"):
    """attention.py:209-267 -> bf16 bits [batch, nq*hd]."""
    return f32_to_bf16_bits(attn_decode_f32(q_bits, kvc, pos, kvs, batch, nq, nkv, hd), mode)


def _l2norm(x, scale=None):
    ss = np.float32(np.sum((x * x).astype(np.float32), dtype=np.float32))
    y = (x * _rsqrt(np.float32(ss + np.float32(1e-6)))).astype(np.float32)
    if scale is not None:
        y = (y * np.float32(scale)).astype(np.float32)
    return y


def delta_decode(qkv_bits, g, beta, state, nh=16, dk=128, dv=128, mode="rne"):
    """linear_attn.py:172-207, one token per batch row b:
    qn = l2norm(q) / sqrt(dk), kn = l2norm(k); S *= exp(g);
    kv = kn^T S; delta = (v - kv) * beta; S += kn delta^T; out = qn^T S.
    qkv [B, 2 nh dk + nh dv] bf16 bits, g / beta [B, nh] fp32, state
    [B*nh, dk, dv] fp32 (updated in place).  Returns out bf16 bits [B, nh*dv]."""
    x = bf16_bits_to_f32(qkv_bits)
    B = x.shape[0]
    g = np.asarray(g, dtype=np.float32).reshape(B, nh)
    beta = np.asarray(beta, dtype=np.float32).reshape(B, nh)
    out = np.empty((B, nh * dv), dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(dk))
    for b in range(B):
        for h in range(nh):
            q = x[b, h * dk:(h + 1) * dk]
            k = x[b, nh * dk + h * dk:nh * dk + (h + 1) * dk]
            v = x[b, 2 * nh * dk + h * dv:2 * nh * dk + (h + 1) * dv]
            qn = _l2norm(q, inv)
            kn = _l2norm(k)
            S = (state[b * nh + h] * np.float32(np.exp(g[b, h]))).astype(np.float32)
            kv = np.sum((kn[:, None] * S).astype(np.float32), axis=0, dtype=np.float32)
            delta = ((v - kv).astype(np.float32) * beta[b, h]).astype(np.float32)
            S = (S + (kn[:, None] * delta[None, :]).astype(np.float32)).astype(np.float32)
            out[b, h * dv:(h + 1) * dv] = np.sum((qn[:, None] * S).astype(np.float32), axis=0, dtype=np.float32)
            state[b * nh + h] = S
    return f32_to_bf16_bits(out, mode)


def conv_silu(x_bits, w_bits, state_bits, T, batch=False, mode="rne"):
    """linear_attn.py:10-47: depthwise causal conv of width KS = w.shape[1]
    then SiLU.  Non-batch: output row t sums x[t - KS + 1 + j] * w[:, j] over
    j (rows before 0 come from the KS - 1 state rows).  Batch: row t is one
    candidate; taps 0..KS-2 read that candidate's state rows t*(KS-1) + j, the
    last tap its own input row.  Returns bf16 bits [T, C]."""
    x = bf16_bits_to_f32(x_bits)
    w = bf16_bits_to_f32(w_bits)
    st = bf16_bits_to_f32(state_bits)
    C, KS = w.shape
    acc = np.zeros((T, C), dtype=np.float32)
    for j in range(KS):
        if batch:
            src = j - (KS - 1)
            xa = x[:T] if src >= 0 else st[np.arange(T) * (KS - 1) + j]
        else:
            rows = np.arange(T) - (KS - 1) + j
            xa = np.where((rows >= 0)[:, None], x[np.clip(rows, 0, None)],
                          st[np.clip(KS - 1 + rows, 0, KS - 2)])
        acc = (acc + (xa * w[None, :, j]).astype(np.float32)).astype(np.float32)
    return f32_to_bf16_bits(silu(acc), mode)


def conv_state_update(x_bits, state_bits, T, batch=1):
    """linear_attn.py:50-83 -> the new state (bf16 bits).  Non-batch: the last
    KS - 1 raw input rows of the T new ones (older ones from the state when T
    is short).  Batch: each candidate's rows shift down by one and take its
    own input row as the newest."""
    x = np.asarray(x_bits, dtype=np.uint16)
    st = np.array(state_bits, dtype=np.uint16, copy=True)
    kk = 3
    if batch > 1:
        for b in range(batch):
            st[b * kk:b * kk + kk - 1] = st[b * kk + 1:b * kk + kk].copy()
            st[b * kk + kk - 1] = x[b]
        return st
    new = st.copy()
    for j in range(kk):
        src = T - kk + j
        new[j] = x[src] if src >= 0 else st[src + kk]
    return new


# ----------------------------------------------------------------------------
# f4: prefill neighbours  (kernels/attention.py:136-206, kernels/linear_attn.py:86-169)
# ----------------------------------------------------------------------------
# ``tl.dot`` is float32 ``np.matmul`` under the CPU interpreter; the
# restatement multiplies blocks of the reference's own shapes the same way.

def _mm(a, b):
    return np.matmul(np.asarray(a, np.float32), np.asarray(b, np.float32), dtype=np.float32)


def attn_prefill(q_bits, kvc, T, pos0=0, kvs=None, nq=8, nkv=2, hd=256, block_m=32, block_n=32, mode="rne"):
    """attention.py:136-206: causal attention of T query rows (positions
    pos0 + t) over cache rows 0 .. pos0 + t.  Per (head, block of block_m
    queries), key blocks of block_n: s = q k^T (bf16 operands; an int8 cache
    is dequantised to bf16(code * scale)), online softmax, acc += bf16(p) v.
    q [T, nq*hd] bf16 bits; kvc [rows, 2*nkv*hd] (bf16 bits or int8, kvs
    fp32).  Returns bf16 bits [T, nq*hd]."""
    q = bf16_bits_to_f32(q_bits)
    out = np.zeros((T, nq * hd), dtype=np.float32)
    sns = 2 * nkv
    for head in range(nq):
        kvh = head // (nq // nkv)
        for mb in range(0, T, block_m):
            rows = np.arange(mb, mb + block_m)
            qb = np.zeros((block_m, hd), dtype=np.float32)
            live = rows < T
            qb[live] = q[rows[live], head * hd:(head + 1) * hd]
            m_i = np.full(block_m, -np.inf, dtype=np.float32)
            l_i = np.zeros(block_m, dtype=np.float32)
            acc = np.zeros((block_m, hd), dtype=np.float32)
            total = pos0 + min(mb + block_m, T)
            for n0 in range(0, total, block_n):
                n = np.arange(n0, n0 + block_n)
                nmask = n < total
                k = np.zeros((block_n, hd), dtype=np.float32)
                v = np.zeros((block_n, hd), dtype=np.float32)
                nv = n[nmask]
                if kvs is None:
                    k[nmask] = bf16_bits_to_f32(kvc[nv, kvh * hd:(kvh + 1) * hd])
                    v[nmask] = bf16_bits_to_f32(kvc[nv, (nkv + kvh) * hd:(nkv + kvh + 1) * hd])
                else:
                    k[nmask] = (kvc[nv, kvh * hd:(kvh + 1) * hd].astype(np.float32) * kvs[nv, kvh][:, None])
                    v[nmask] = (kvc[nv, (nkv + kvh) * hd:(nkv + kvh + 1) * hd].astype(np.float32)
                                * kvs[nv, nkv + kvh][:, None])
                    k, v = bf16_round(k, mode), bf16_round(v, mode)
                sc = _mm(qb, k.T)
                causal = ((pos0 + rows)[:, None] >= n[None, :]) & nmask[None, :]
                sc = np.where(causal, sc, np.float32(-np.inf)).astype(np.float32)
                m_new = np.maximum(m_i, sc.max(axis=1)).astype(np.float32)
                with np.errstate(invalid="ignore"):
                    p = np.exp((sc - m_new[:, None]).astype(np.float32)).astype(np.float32)
                    alpha = np.exp((m_i - m_new).astype(np.float32)).astype(np.float32)
                l_i = ((l_i * alpha).astype(np.float32) + np.sum(p, axis=1, dtype=np.float32)).astype(np.float32)
                acc = (acc * alpha[:, None]).astype(np.float32)
                acc = (acc + _mm(bf16_round(p, mode), v)).astype(np.float32)
                m_i = m_new
            l_safe = np.where(l_i > 0, l_i, np.float32(1.0)).astype(np.float32)
            res = (acc / l_safe[:, None]).astype(np.float32)
            out[rows[live], head * hd:(head + 1) * hd] = res[live]
    return f32_to_bf16_bits(out, mode)


def _ut_inverse(A):
    """linear_attn.py:86-95: (I - A)^-1 for strictly lower A by the Neumann
    product: Tm = I + A, P = A; five times P = P P, Tm = Tm + Tm P."""
    C = A.shape[0]
    eye = np.eye(C, dtype=np.float32)
    Tm = (eye + A).astype(np.float32)
    P = A
    for _ in range(5):
        P = _mm(P, P)
        Tm = (Tm + _mm(Tm, P)).astype(np.float32)
    return Tm


def delta_prefill(qkv_bits, g, beta, state, T, nh=16, dk=128, dv=128, vs=32, chunk=32, mode="rne"):
    """linear_attn.py:98-169: chunked gated delta rule over T tokens, per head
    and per vs-column slab of the state (grid (NH, DV/VS)), chunks of 32 in
    order.  qkv [T, 2 nh dk + nh dv] bf16 bits, g / beta [T, nh] fp32, state
    [nh, dk, dv] fp32 (updated in place).  Returns out bf16 bits [T, nh*dv]."""
    x = bf16_bits_to_f32(qkv_bits)
    g = np.asarray(g, np.float32)
    beta = np.asarray(beta, np.float32)
    out = np.zeros((T, nh * dv), dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(dk))
    c = np.arange(chunk)
    for h in range(nh):
        for slab in range(dv // vs):
            cols = slice(slab * vs, (slab + 1) * vs)
            S = state[h][:, cols].astype(np.float32).copy()
            for c0 in range(0, T, chunk):
                t = c0 + c
                live = t < T
                tl_ = t[live]
                q = np.zeros((chunk, dk), np.float32)
                k = np.zeros((chunk, dk), np.float32)
                v = np.zeros((chunk, vs), np.float32)
                q[live] = x[tl_, h * dk:(h + 1) * dk]
                k[live] = x[tl_, nh * dk + h * dk:nh * dk + (h + 1) * dk]
                v[live] = x[tl_, 2 * nh * dk + h * dv:2 * nh * dk + (h + 1) * dv][:, cols]
                bt = np.zeros(chunk, np.float32)
                gg = np.zeros(chunk, np.float32)
                bt[live] = beta[tl_, h]
                gg[live] = g[tl_, h]
                sq = np.sum((q * q).astype(np.float32), axis=1, keepdims=True, dtype=np.float32)
                sk = np.sum((k * k).astype(np.float32), axis=1, keepdims=True, dtype=np.float32)
                qn = ((q * _rsqrt((sq + np.float32(1e-6)).astype(np.float32))).astype(np.float32) * inv).astype(
                    np.float32)
                kn = (k * _rsqrt((sk + np.float32(1e-6)).astype(np.float32))).astype(np.float32)
                gc = np.cumsum(gg, dtype=np.float32)
                with np.errstate(over="ignore"):
                    decay = np.where(c[:, None] >= c[None, :],
                                     np.exp((gc[:, None] - gc[None, :]).astype(np.float32)), np.float32(0.0))
                decay = decay.astype(np.float32)
                kb = (kn * bt[:, None]).astype(np.float32)
                A = (-_mm(kb, kn.T) * decay).astype(np.float32)
                A = np.where(c[:, None] > c[None, :], A, np.float32(0.0)).astype(np.float32)
                Tm = _ut_inverse(A)
                vb = (v * bt[:, None]).astype(np.float32)
                value = _mm(Tm, vb)
                eg = np.exp(gc).astype(np.float32)
                kcum = _mm(Tm, (kb * eg[:, None]).astype(np.float32))
                v_new = (value - _mm(kcum, S)).astype(np.float32)
                o = _mm((qn * eg[:, None]).astype(np.float32), S)
                o = (o + _mm((_mm(qn, kn.T) * decay).astype(np.float32), v_new)).astype(np.float32)
                g_last = np.float32(np.min(gc))
                w = (kn * np.exp((g_last - gc).astype(np.float32))[:, None]).astype(np.float32)
                S = ((S * np.float32(np.exp(g_last))).astype(np.float32) + _mm(w.T, v_new)).astype(np.float32)
                out[tl_, h * dv + slab * vs:h * dv + (slab + 1) * vs] = o[live]
            state[h][:, cols] = S
    return f32_to_bf16_bits(out, mode)


# ----------------------------------------------------------------------------
# CPU baseline: the reference's own dequant-then-matmul (.dev/test_kernels.py:40-41)
# ----------------------------------------------------------------------------

def dequant_matmul_w8(a_q, a_s, b, b_s):
    """``(a_q.float() * a_s.repeat_interleave(64, 1)) @ b.float() * b_s`` (torch, CPU)."""
    import torch
    af = a_q.float() * a_s.repeat_interleave(GROUP, dim=1)
    return (af @ b.float()) * b_s[None, :]


def dequant_matmul_w4(a_q, a_s, b, b_s, b_z=None):
    """The W4 analogue: dequantise ``(nibble - z) * scale`` then one fp32 matmul."""
    import torch
    K2, N = b.shape
    K = 2 * K2
    wgrp = K // b_s.shape[0]
    nib = torch.empty((K, N), dtype=torch.int16)
    nib[0::2] = (b & 0x0F).to(torch.int16)
    nib[1::2] = (b >> 4).to(torch.int16)
    z = torch.full((1, 1), 8, dtype=torch.int16) if b_z is None else b_z.to(torch.int16).repeat_interleave(wgrp, 0)
    w = (nib - z).float() * b_s.float().repeat_interleave(wgrp, 0)
    af = a_q.float() * a_s.repeat_interleave(GROUP, dim=1)
    return af @ w
