"""Generate golden input/output vectors by running the reference kernels on CPU.

The reference's Triton kernels (``kernels/gemm.py``, ``kernels/w4.py``,
``kernels/norm.py``) run on the CPU under Triton's interpreter
(``TRITON_INTERPRET=1``).  This script imports them from a read-only checkout of
the reference project, runs every hot-path entry point on small seeded inputs
and stores inputs and outputs in ``ref_golden.npz`` (GEMMs, quant_row) and
``ref_golden_norm.npz`` (the other activation producers) and
``ref_golden_decode.npz`` (the decode-step neighbours of kernels/attention.py
and kernels/linear_attn.py) next to this file.

The interpreter converts fp32 -> bf16 by truncation (a GPU build rounds to
nearest-even), so the fixtures pin the oracle in its ``mode="trunc"``; every
other step of the arithmetic is shared by both modes.

Usage (in a container that has the reference checkout)::

    python tests/golden/make_golden.py /path/to/reference [gemm|norm|decode|all]

bf16 tensors are stored as uint16 bit patterns.  Nothing at test time reads
the reference: the tests only load the committed ``.npz``.
"""
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"
sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "ref_golden.npz")


def import_reference(root):
    """Register the reference checkout as package ``qwen35_prompt_enhancer``
    without executing its ``__init__`` (which pulls in the ComfyUI node)."""
    pkg = types.ModuleType("qwen35_prompt_enhancer")
    pkg.__path__ = [root]
    sys.modules["qwen35_prompt_enhancer"] = pkg
    from qwen35_prompt_enhancer.kernels import gemm, norm, w4  # noqa: F401
    return gemm, w4, norm


def bits(t):
    """bf16 torch tensor -> uint16 numpy bit pattern."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def producers(norm):
    """Activation producers of kernels/norm.py -> ref_golden_norm.npz."""
    G = 64
    rec = {}

    def bf(t):
        return t.to(torch.bfloat16)

    # rmsnorm_quant (norm.py:28-57): K a power of two, K padded inside the
    # reference's block (1088 -> 2048), a strided x, one_plus on/off,
    # outliers and an all-zero row
    for i, (M, K, one_plus, strided) in enumerate([(3, 256, True, False), (4, 2048, True, True),
                                                    (2, 1088, False, False)]):
        g = torch.Generator().manual_seed(900 + i)
        xw = torch.randn(M, K + (64 if strided else 0), generator=g)
        xw[torch.rand(xw.shape, generator=g) < 0.002] *= 20.0
        xw[-1] = 0.0 if M > 2 else xw[-1]
        xb = bf(xw)
        x = xb[:, :K]
        w = bf(torch.randn(K, generator=g) * 0.2)
        q = torch.empty(M, K, dtype=torch.int8)
        s = torch.empty(M, K // G, dtype=torch.float32)
        norm.rmsnorm_quant(x, w, q, s, 1e-6, one_plus)
        p = f"rmsnorm_quant_{i}_"
        rec[p + "x"] = bits(x.contiguous()); rec[p + "w"] = bits(w)
        rec[p + "one_plus"] = np.array(int(one_plus)); rec[p + "q"] = q.numpy(); rec[p + "s"] = s.numpy()

    # norm_gated_quant / norm_gated (norm.py:95-165): HD = 128 and 64, z a
    # column slice of a wider projection row (engine.py:230-231)
    for i, (T, NV, HD) in enumerate([(3, 16, 128), (2, 2, 256)]):
        g = torch.Generator().manual_seed(950 + i)
        N = NV * HD
        v = bf(torch.randn(T, N, generator=g) * 0.7)
        proj = bf(torch.randn(T, N + 96, generator=g))
        z = proj[:, 96:]
        w = bf(torch.randn(HD, generator=g) * 0.3 + 1.0)
        q = torch.empty(T, N, dtype=torch.int8)
        s = torch.empty(T, N // G, dtype=torch.float32)
        norm.norm_gated_quant(v, z, w, q, s, 1e-6)
        o = torch.empty(T, N, dtype=torch.bfloat16)
        norm.norm_gated(v, z, w, o, 1e-6)
        p = f"norm_gated_{i}_"
        rec[p + "v"] = bits(v); rec[p + "z"] = bits(z.contiguous()); rec[p + "w"] = bits(w)
        rec[p + "q"] = q.numpy(); rec[p + "s"] = s.numpy(); rec[p + "out"] = bits(o)

    # gate_mul_quant (norm.py:168-188): the q projection row holds (q, gate)
    # halves per head and is wider than 2N (engine.py:262)
    for i, (M, NQ, HD) in enumerate([(3, 8, 256), (2, 2, 128)]):
        g = torch.Generator().manual_seed(970 + i)
        N = NQ * HD
        a = bf(torch.randn(M, N, generator=g))
        proj = bf(torch.randn(M, 2 * N + 128, generator=g) * 2.0)
        q = torch.empty(M, N, dtype=torch.int8)
        s = torch.empty(M, N // G, dtype=torch.float32)
        norm.gate_mul_quant(a, proj, q, s, hd=HD)
        p = f"gate_mul_quant_{i}_"
        rec[p + "a"] = bits(a); rec[p + "g"] = bits(proj); rec[p + "hd"] = np.array(HD)
        rec[p + "q"] = q.numpy(); rec[p + "s"] = s.numpy()

    # silu_mul_quant (norm.py:191-208)
    g = torch.Generator().manual_seed(980)
    gg = bf(torch.randn(2, 512, generator=g) * 2.0)
    uu = bf(torch.randn(2, 512, generator=g))
    q = torch.empty(2, 512, dtype=torch.int8)
    s = torch.empty(2, 512 // G, dtype=torch.float32)
    norm.silu_mul_quant(gg, uu, q, s)
    rec["silu_mul_quant_0_g"] = bits(gg); rec["silu_mul_quant_0_u"] = bits(uu)
    rec["silu_mul_quant_0_q"] = q.numpy(); rec["silu_mul_quant_0_s"] = s.numpy()

    # gate_proj (norm.py:211-240), .dev/test_kernels.py:83-99 distributions,
    # K a power of two and a padded K
    for i, (M, K, NB) in enumerate([(5, 2048, 16), (2, 320, 16)]):
        g = torch.Generator().manual_seed(990 + i)
        a = torch.randint(-127, 127, (M, K), dtype=torch.int8, generator=g)
        a_s = torch.rand(M, K // G, generator=g) * 0.02
        wb = bf(torch.randn(NB, K, generator=g) * 0.05)
        wa = bf(torch.randn(NB, K, generator=g) * 0.05)
        dt = bf(torch.randn(NB, generator=g))
        al = bf(torch.randn(NB, generator=g))
        beta = torch.empty(M, NB)
        gate = torch.empty(M, NB)
        norm.gate_proj(a, a_s, wb, wa, beta, gate, dt, al)
        p = f"gate_proj_{i}_"
        rec[p + "a"] = a.numpy(); rec[p + "as"] = a_s.numpy(); rec[p + "wb"] = bits(wb); rec[p + "wa"] = bits(wa)
        rec[p + "dt"] = bits(dt); rec[p + "alog"] = bits(al)
        rec[p + "beta"] = beta.numpy(); rec[p + "gate"] = gate.numpy()

    out = os.path.join(HERE, "ref_golden_norm.npz")
    np.savez_compressed(out, **rec)
    print(f"wrote {out}: {len(rec)} arrays, {os.path.getsize(out)} bytes")


def _widen_bf16_dot_operands():
    """Triton 3.6's CPU interpreter stores bf16 tensors as their uint16 bit
    patterns and its ``tl.dot`` multiplies that storage as integers, so any
    dot with bf16 operands (attn_prefill's q k^T and p v) comes out as
    garbage.  Widen such operands to fp32 first -- exact for bf16 -- which is
    what a bf16 MMA with fp32 accumulation computes.  The reference's code is
    untouched; only the interpreter's dot is corrected."""
    import triton.language as tl
    from triton.runtime import interpreter as interp
    orig = interp.InterpreterBuilder.create_dot
    if getattr(orig, "_widened", False):
        return

    def widen(h):
        if h.dtype.scalar == tl.bfloat16:
            return interp.TensorHandle((h.data.astype(np.uint32) << 16).view(np.float32), tl.float32)
        return h

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        return orig(self, widen(a), widen(b), d, input_precision, max_num_imprecise_acc)
    create_dot._widened = True
    interp.InterpreterBuilder.create_dot = create_dot


def neighbours():
    """Decode-step neighbours of kernels/attention.py and kernels/linear_attn.py
    -> ref_golden_decode.npz."""
    from qwen35_prompt_enhancer.kernels import attention, linear_attn
    _widen_bf16_dot_operands()
    rec = {}

    def bf(t):
        return t.to(torch.bfloat16)

    NQ, NKV, HD, RD = 8, 2, 256, 64
    invf = 1.0 / (1e7 ** (torch.arange(0, RD, 2, dtype=torch.float32) / RD))
    P = NQ * HD * 2 + 2 * NKV * HD
    # qk_norm_rope (attention.py:70-133): sequence mode (positions pos0 + t)
    # with bf16 and int8 caches, and batch mode (candidates at one position)
    for i, (T, pos0, int8, batch) in enumerate([(3, 5, False, False), (3, 5, True, False), (2, 1030, True, True)]):
        g = torch.Generator().manual_seed(1700 + i)
        proj = bf(torch.randn(T, P + 64, generator=g) * 0.5)
        qn = bf(torch.randn(HD, generator=g) * 0.2)
        kn = bf(torch.randn(HD, generator=g) * 0.2)
        seq = pos0 + T + 4
        rows = T * seq if batch else seq
        kvc = torch.zeros(rows, 2 * NKV * HD, dtype=torch.int8 if int8 else torch.bfloat16)
        kvs = torch.zeros(rows, 2 * NKV) if int8 else None
        qout = torch.empty(T, NQ * HD, dtype=torch.bfloat16)
        attention.qk_norm_rope(proj, qn, kn, invf, qout, kvc, kvs, pos0, 1e-6, kv_int8=int8, batch=batch,
                               kv_stride=seq * 2 * NKV * HD if batch else None,
                               kvs_stride=seq * 2 * NKV if batch else None)
        p = f"qk_rope_{i}_"
        rec[p + "proj"] = bits(proj); rec[p + "qn"] = bits(qn); rec[p + "kn"] = bits(kn)
        rec[p + "invf"] = invf.numpy(); rec[p + "cfg"] = np.array([T, pos0, int(int8), int(batch), seq])
        rec[p + "q"] = bits(qout)
        rec[p + "kvc"] = kvc.numpy() if int8 else bits(kvc)
        if int8:
            rec[p + "kvs"] = kvs.numpy()

    # attn_decode (attention.py:209-267): bf16 / int8 caches, batch 1 and 3,
    # positions that end inside and on a 32-position block
    for i, (B, pos, int8) in enumerate([(1, 40, False), (1, 63, True), (3, 70, True)]):
        g = torch.Generator().manual_seed(1750 + i)
        S = pos + 9
        q = bf(torch.randn(B, NQ * HD, generator=g) * 0.1)
        if int8:
            kvc = torch.randint(-127, 128, (B * S, 2 * NKV * HD), dtype=torch.int8, generator=g)
            kvs = torch.rand(B * S, 2 * NKV, generator=g) * 0.02 + 0.001
        else:
            kvc = bf(torch.randn(B * S, 2 * NKV * HD, generator=g))
            kvs = None
        out = torch.empty(B, NQ * HD, dtype=torch.bfloat16)
        attention.attn_decode(q if B > 1 else q[0], kvc, out if B > 1 else out[0], pos, kvs=kvs, kv_int8=int8,
                              batch=B, nq=NQ, nkv=NKV, hd=HD)
        p = f"attn_decode_{i}_"
        rec[p + "q"] = bits(q); rec[p + "cfg"] = np.array([B, pos, int(int8)])
        rec[p + "kvc"] = kvc.numpy() if int8 else bits(kvc)
        if int8:
            rec[p + "kvs"] = kvs.numpy()
        rec[p + "out"] = bits(out)

    # delta_decode (linear_attn.py:172-207), .dev/test_kernels.py:151-163 distributions
    NH, DK, DV = 16, 128, 128
    C = 2 * NH * DK + NH * DV
    for i, B in enumerate([1, 2]):
        g = torch.Generator().manual_seed(1800 + i)
        qkv = bf(torch.randn(B, C, generator=g) * 0.3)
        gg = -torch.rand(B, NH, generator=g) * 0.4
        beta = torch.rand(B, NH, generator=g)
        # state values on a 2^-8 grid (|s| <= 0.0625): exact in fp32 and
        # compressible; the output state is stored for two heads only
        state = torch.randint(-16, 17, (B * NH, DK, DV), generator=g).float() / 256.0
        st = state.clone()
        out = torch.empty(B, NH * DV, dtype=torch.bfloat16)
        if B == 1:
            linear_attn.delta_decode(qkv[0], gg[0], beta[0], st, out[0])
        else:
            linear_attn.delta_decode(qkv, gg, beta, st, out, batch=B)
        p = f"delta_decode_{i}_"
        rec[p + "qkv"] = bits(qkv); rec[p + "g"] = gg.numpy(); rec[p + "beta"] = beta.numpy()
        rec[p + "state"] = state.numpy(); rec[p + "state_out2"] = st[:2].numpy(); rec[p + "out"] = bits(out)

    # conv_silu / conv_state_update (linear_attn.py:10-83), test_kernels.py:166-184 shapes
    for i, (T, batch, Cc) in enumerate([(23, False, 2048), (1, False, 512), (3, True, C)]):
        g = torch.Generator().manual_seed(1850 + i)
        x = bf(torch.randn(T, Cc, generator=g))
        w = bf(torch.randn(Cc, 4, generator=g) * 0.1)
        state = bf(torch.randn(3 * T if batch else 3, Cc, generator=g))
        y = torch.empty(T, Cc, dtype=torch.bfloat16)
        linear_attn.conv_silu(x, w, state, y, T, batch=batch)
        st2 = state.clone()
        linear_attn.conv_state_update(x, st2, T, batch=T if batch else 1)
        p = f"conv_{i}_"
        rec[p + "x"] = bits(x); rec[p + "w"] = bits(w); rec[p + "state"] = bits(state)
        rec[p + "cfg"] = np.array([T, int(batch)]); rec[p + "y"] = bits(y); rec[p + "state_out"] = bits(st2)

    # attn_prefill (attention.py:136-206): one chunk from position 0 and a
    # later chunk over an earlier one, bf16 and int8 caches
    for i, (T, pos0, int8) in enumerate([(40, 0, False), (19, 37, True)]):
        g = torch.Generator().manual_seed(1900 + i)
        q = bf(torch.randn(T, NQ * HD, generator=g) * 0.1)
        S = pos0 + T + 5
        if int8:
            kvc = torch.randint(-127, 128, (S, 2 * NKV * HD), dtype=torch.int8, generator=g)
            kvs = torch.rand(S, 2 * NKV, generator=g) * 0.02 + 0.001
        else:
            kvc = bf(torch.randn(S, 2 * NKV * HD, generator=g))
            kvs = None
        out = torch.empty(T, NQ * HD, dtype=torch.bfloat16)
        attention.attn_prefill(q, kvc, out, T, pos0, kvs=kvs, kv_int8=int8, nq=NQ, nkv=NKV, hd=HD)
        p = f"attn_prefill_{i}_"
        rec[p + "q"] = bits(q); rec[p + "cfg"] = np.array([T, pos0, int(int8)])
        rec[p + "kvc"] = kvc.numpy() if int8 else bits(kvc)
        if int8:
            rec[p + "kvs"] = kvs.numpy()
        rec[p + "out"] = bits(out)

    # delta_prefill (linear_attn.py:98-169), test_kernels.py:151-163 distributions:
    # a partial chunk and a run over two chunks plus a partial one
    for i, T in enumerate([5, 70]):
        g = torch.Generator().manual_seed(1950 + i)
        qkv = bf(torch.randn(T, C, generator=g) * 0.3)
        gg = -torch.rand(T, NH, generator=g) * 0.4
        beta = torch.rand(T, NH, generator=g)
        state = torch.randint(-16, 17, (NH, DK, DV), generator=g).float() / 256.0
        st = state.clone()
        out = torch.empty(T, NH * DV, dtype=torch.bfloat16)
        linear_attn.delta_prefill(qkv, gg, beta, st, out, T)
        p = f"delta_prefill_{i}_"
        rec[p + "qkv"] = bits(qkv); rec[p + "g"] = gg.numpy(); rec[p + "beta"] = beta.numpy()
        rec[p + "state"] = state.numpy(); rec[p + "state_out2"] = st[:2].numpy(); rec[p + "out"] = bits(out)

    out = os.path.join(HERE, "ref_golden_decode.npz")
    np.savez_compressed(out, **rec)
    print(f"wrote {out}: {len(rec)} arrays, {os.path.getsize(out)} bytes")


def main():
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: make_golden.py /path/to/reference-checkout [gemm|norm|decode|all]")
    root = sys.argv[1]
    which = sys.argv[2] if len(sys.argv) == 3 else "all"
    gemm, w4, norm = import_reference(root)
    if which in ("norm", "all"):
        producers(norm)
    if which in ("decode", "all"):
        neighbours()
    if which in ("norm", "decode"):
        return
    G = 64
    rec = {}

    def gen(seed):
        g = torch.Generator().manual_seed(seed)
        return g

    def act(g, M, K, dist="ref"):
        if dist == "ref":   # .dev/test_kernels.py:34-36
            a = torch.randint(-127, 127, (M, K), dtype=torch.int8, generator=g)
            s = torch.rand(M, K // G, generator=g) * 0.02
            return a, s
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        q = torch.empty(M, K, dtype=torch.int8)
        s = torch.empty(M, K // G, dtype=torch.float32)
        norm.quant_row(x, q, s)
        return q, s

    def w8(g, K, N):
        b = torch.randint(-127, 127, (K, N), dtype=torch.int8, generator=g)
        bs = torch.rand(N, generator=g) * 0.002
        return b, bs

    def w4w(g, K, N, wg, zeros):
        b = torch.randint(0, 256, (K // 2, N), dtype=torch.int32, generator=g).to(torch.uint8)
        s = torch.exp(torch.randn(K // wg, N, generator=g) * 0.5 - 5.0).to(torch.bfloat16)
        z = torch.randint(0, 16, (K // wg, N), dtype=torch.int32, generator=g).to(torch.uint8) if zeros else None
        return b, s, z

    # ---------------- a9: quant_row (norm.py:75-92), incl. outliers and zero groups
    for i, (M, K) in enumerate([(3, 256), (5, 2048)]):
        g = gen(100 + i)
        x = torch.randn(M, K, generator=g)
        x[torch.rand(M, K, generator=g) < 0.01] *= 20.0
        x[0, 64:128] = 0.0                       # all-zero group -> scale 1e-8
        x[-1, :4] = torch.tensor([0.5, -0.5, 1e-30, -3.0])
        x = x.to(torch.bfloat16)
        q = torch.empty(M, K, dtype=torch.int8)
        s = torch.empty(M, K // G, dtype=torch.float32)
        norm.quant_row(x, q, s)
        p = f"quant_row_{i}_"
        rec[p + "x"] = bits(x)
        rec[p + "q"] = q.numpy()
        rec[p + "s"] = s.numpy()

    # ---------------- a1: gemm_i8 (gemm.py:60-92)
    cases = [
        (1, 192, 256, False, "ref"),
        (4, 320, 512, True, "ref"),
        (5, 208, 128, True, "x"),      # ragged N (not a multiple of the tile), quant_row acts
        (37, 128, 256, False, "ref"),  # M > 16 -> reference's larger tile path
    ]
    for i, (M, N, K, res, dist) in enumerate(cases):
        g = gen(200 + i)
        a, s = act(g, M, K, dist)
        b, bs = w8(g, K, N)
        p = f"gemm_i8_{i}_"
        if res:
            # out is a row-slice of a wider buffer and aliases the residual,
            # exactly as the engine calls it (engine.py:238-240).
            buf = torch.randn(M, N + 48, generator=g).to(torch.bfloat16)
            rec[p + "res"] = bits(buf[:, :N])
            out = buf[:, :N]
            gemm.gemm_i8(a, s, b, bs, out, residual=out)
        else:
            out = torch.empty(M, N, dtype=torch.bfloat16)
            gemm.gemm_i8(a, s, b, bs, out)
        rec[p + "a"] = a.numpy(); rec[p + "as"] = s.numpy()
        rec[p + "b"] = b.numpy(); rec[p + "bs"] = bs.numpy()
        rec[p + "out"] = bits(out)

    # ---------------- a5: gemm_w4 (w4.py:139-166), groups 32/64/128, zeros on/off
    cases = [
        (1, 128, 256, 128, True, False),
        (4, 192, 256, 64, False, True),
        (3, 128, 256, 32, True, True),
        (2, 256, 512, 256, True, False),
    ]
    for i, (M, N, K, wg, zeros, res) in enumerate(cases):
        g = gen(300 + i)
        a, s = act(g, M, K, "x")
        b, bsc, bz = w4w(g, K, N, wg, zeros)
        p = f"gemm_w4_{i}_"
        out = torch.empty(M, N, dtype=torch.bfloat16)
        r = None
        if res:
            r = torch.randn(M, N, generator=g).to(torch.bfloat16)
            rec[p + "res"] = bits(r)
        w4.gemm_w4(a, s, b, bsc, out, residual=r, b_z=bz)
        rec[p + "a"] = a.numpy(); rec[p + "as"] = s.numpy()
        rec[p + "b"] = b.numpy(); rec[p + "bs"] = bits(bsc)
        if bz is not None:
            rec[p + "bz"] = bz.numpy()
        rec[p + "out"] = bits(out)

    # ---------------- a2: proj3 W8 (gemm.py:290-312), out wider than N1+N2+N3
    for i, (M, K, ns) in enumerate([(2, 256, (192, 64, 64)), (3, 128, (128, 64, 0))]):
        g = gen(400 + i)
        a, s = act(g, M, K, "ref")
        ws = [w8(g, K, n) if n else (None, None) for n in ns]
        out = torch.zeros(M, sum(ns) + 64, dtype=torch.bfloat16)
        gemm.proj3(a, s, ws[0][0], ws[0][1], ws[1][0], ws[1][1], ws[2][0], ws[2][1], out)
        p = f"proj3_{i}_"
        rec[p + "a"] = a.numpy(); rec[p + "as"] = s.numpy()
        for j, (w, sc) in enumerate(ws):
            if w is not None:
                rec[p + f"w{j}"] = w.numpy(); rec[p + f"s{j}"] = sc.numpy()
        rec[p + "out"] = bits(out)

    # ---------------- a6: proj3_w4 (w4.py:220-251)
    for i, (M, K, ns, wg, zeros) in enumerate([(1, 256, (128, 64, 64), 128, True),
                                                (4, 256, (192, 64, 0), 64, False)]):
        g = gen(500 + i)
        a, s = act(g, M, K, "x")
        ws = [w4w(g, K, n, wg, zeros) if n else (None, None, None) for n in ns]
        out = torch.zeros(M, sum(ns) + 32, dtype=torch.bfloat16)
        w4.proj3_w4(a, s, ws[0][0], ws[0][1], ws[1][0], ws[1][1], ws[2][0], ws[2][1], out,
                    z1=ws[0][2], z2=ws[1][2], z3=ws[2][2])
        p = f"proj3_w4_{i}_"
        rec[p + "a"] = a.numpy(); rec[p + "as"] = s.numpy()
        for j, (w, sc, z) in enumerate(ws):
            if w is not None:
                rec[p + f"w{j}"] = w.numpy(); rec[p + f"s{j}"] = bits(sc)
                if z is not None:
                    rec[p + f"z{j}"] = z.numpy()
        rec[p + "out"] = bits(out)

    # ---------------- a4 / a3: mlp_gate_up (bf16) and mlp_gate_up_quant (gemm.py:140-231)
    for i, (M, K, N) in enumerate([(1, 256, 192), (5, 128, 128)]):
        g = gen(600 + i)
        a, s = act(g, M, K, "ref")
        wg_, sg = w8(g, K, N)
        wu_, su = w8(g, K, N)
        h = torch.empty(M, N, dtype=torch.bfloat16)
        gemm.mlp_gate_up(a, s, wg_, sg, wu_, su, h)
        q = torch.empty(M, N, dtype=torch.int8)
        qs = torch.empty(M, N // G, dtype=torch.float32)
        gemm.mlp_gate_up_quant(a, s, wg_, sg, wu_, su, q, qs)
        p = f"gate_up_{i}_"
        rec[p + "a"] = a.numpy(); rec[p + "as"] = s.numpy()
        rec[p + "wg"] = wg_.numpy(); rec[p + "sg"] = sg.numpy()
        rec[p + "wu"] = wu_.numpy(); rec[p + "su"] = su.numpy()
        rec[p + "h"] = bits(h); rec[p + "q"] = q.numpy(); rec[p + "qs"] = qs.numpy()

    # ---------------- a7: mlp_gate_up_quant_w4 (w4.py:300-323)
    for i, (M, K, N, wg, zeros) in enumerate([(1, 256, 128, 128, True), (4, 256, 192, 64, False),
                                               (2, 128, 128, 32, True)]):
        g = gen(700 + i)
        a, s = act(g, M, K, "x")
        wgt, sg, zg = w4w(g, K, N, wg, zeros)
        wut, su, zu = w4w(g, K, N, wg, zeros)
        q = torch.empty(M, N, dtype=torch.int8)
        qs = torch.empty(M, N // G, dtype=torch.float32)
        w4.mlp_gate_up_quant_w4(a, s, wgt, sg, wut, su, q, qs, zg=zg, zu=zu)
        p = f"gate_up_w4_{i}_"
        rec[p + "a"] = a.numpy(); rec[p + "as"] = s.numpy()
        rec[p + "wg"] = wgt.numpy(); rec[p + "sg"] = bits(sg)
        rec[p + "wu"] = wut.numpy(); rec[p + "su"] = bits(su)
        if zeros:
            rec[p + "zg"] = zg.numpy(); rec[p + "zu"] = zu.numpy()
        rec[p + "q"] = q.numpy(); rec[p + "qs"] = qs.numpy()

    np.savez_compressed(OUT, **rec)
    print(f"wrote {OUT}: {len(rec)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
