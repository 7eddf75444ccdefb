"""Activation producers (kernels/norm.py) on the CUDA path against the CPU
oracle and against the reference's own outputs (golden fixtures).

Parity rules, by what each producer computes:

* rmsnorm_quant, gate_mul_quant, silu_mul_quant quantise an fp32 value y.
  The kernel's fp32 sums (rmsnorm) and its library expf (sigmoid) may differ
  from the reference in the last bits of y, and that can only move an int8
  code across a rounding boundary.  So: scales within 4e-6 relative, and
  every code equal except where the oracle's y / s lies within 1e-4 of a
  .5 boundary, where it may differ by one.
* norm_gated_quant rounds y through bf16 before quantising, so a last-bit
  difference can move y by one bf16 step: the fused-quantisation rule of the
  reference's own test (test_fused.py:43-46) -- >= 99.9 % of codes equal, all
  within +-1, scales within 1 % -- as for mlp_gate_up_quant.
* norm_gated's bf16 output: |d| <= 1e-3 + 1e-2 |ref| elementwise.
* gate_proj's fp32 outputs: |d| <= 1e-5 + 1e-4 |ref| (sums of K products in
  another order).
"""
import os

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O
from qlin_testutil import assert_bf16_close, assert_quant_close, bits, from_bits

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden_norm.npz"))


def assert_codes_near_ties(q, s, y, what):
    """q, s from the GPU; y the oracle's fp32 values that were quantised."""
    rq, rs = O.quant_groups(y)
    np.testing.assert_allclose(s, rs, rtol=4e-6, atol=0, err_msg=f"{what}: scales")
    d = q.astype(np.int32) - rq.astype(np.int32)
    if not d.any():
        return
    M, K = y.shape
    v = np.abs(y.reshape(M, K // 64, 64) / rs[:, :, None]).reshape(M, K)
    near = np.abs(v - np.floor(v) - 0.5) < 1e-4
    bad = (d != 0) & ~(near & (np.abs(d) == 1))
    assert not bad.any(), f"{what}: {int(bad.sum())} codes differ away from a rounding tie"


def bf16_t(a, dev):
    return from_bits(a).to(dev)


def rand_bf16(g, shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


# ---------------------------------------------------------------- rmsnorm_quant
@pytest.mark.parametrize("M,K,one_plus,strided", [(1, 2048, True, False), (4, 2048, True, True),
                                                  (37, 1024, False, False), (512, 2048, True, False),
                                                  (3, 6144, True, False), (2, 64, True, False)])
def test_rmsnorm_quant_vs_oracle(pkg, dev, M, K, one_plus, strided):
    g = torch.Generator().manual_seed(1100 + M + K)
    xw = torch.randn(M, K + (128 if strided else 0), generator=g)
    xw[torch.rand(xw.shape, generator=g) < 0.001] *= 20.0
    xb = xw.to(torch.bfloat16)
    w = rand_bf16(g, (K,), 0.2)
    xd = xb.to(dev)[:, :K]
    q = torch.empty(M, K, dtype=torch.int8, device=dev)
    s = torch.empty(M, K // 64, dtype=torch.float32, device=dev)
    rq, rs = pkg.rmsnorm_quant(xd, w.to(dev), q, s, 1e-6, one_plus)
    assert rq is q and rs is s
    y = O.rmsnorm_y(bits(xb[:, :K]), bits(w), 1e-6, one_plus)
    assert_codes_near_ties(q.cpu().numpy(), s.cpu().numpy(), y, f"rmsnorm_quant M={M} K={K}")


@pytest.mark.parametrize("i", ["0", "1"])
def test_rmsnorm_quant_vs_reference_golden(pkg, dev, i):
    p = f"rmsnorm_quant_{i}_"
    x, w = GOLD[p + "x"], GOLD[p + "w"]
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.int8, device=dev)
    s = torch.empty(M, K // 64, dtype=torch.float32, device=dev)
    pkg.rmsnorm_quant(bf16_t(x, dev), bf16_t(w, dev), q, s, 1e-6, bool(GOLD[p + "one_plus"]))
    y = O.rmsnorm_y(x, w, 1e-6, bool(GOLD[p + "one_plus"]))
    np.testing.assert_array_equal(O.quant_groups(y)[0], GOLD[p + "q"])  # the oracle is the reference here
    assert_codes_near_ties(q.cpu().numpy(), s.cpu().numpy(), y, f"rmsnorm_quant golden {i}")


def test_rmsnorm_quant_zero_row(pkg, dev):
    """An all-zero row: var = 0, y = 0, every scale 1e-8 and every code 0."""
    x = torch.zeros(2, 256, dtype=torch.bfloat16, device=dev)
    q = torch.full((2, 256), 5, dtype=torch.int8, device=dev)
    s = torch.empty(2, 4, dtype=torch.float32, device=dev)
    pkg.rmsnorm_quant(x, torch.ones(256, dtype=torch.bfloat16, device=dev), q, s)
    assert (q == 0).all() and torch.equal(s, torch.full_like(s, 1e-8))


# ---------------------------------------------------------------- norm_gated(_quant)
@pytest.mark.parametrize("T,NV,HD,zpad", [(1, 16, 128, 0), (4, 16, 128, 2048), (33, 16, 128, 64),
                                          (3, 2, 256, 0), (5, 8, 64, 32)])
def test_norm_gated_vs_oracle(pkg, dev, T, NV, HD, zpad):
    g = torch.Generator().manual_seed(1200 + T + HD)
    N = NV * HD
    v = rand_bf16(g, (T, N), 0.7)
    zw = rand_bf16(g, (T, zpad + N))
    w = (torch.randn(HD, generator=g) * 0.3 + 1.0).to(torch.bfloat16)
    zd = zw.to(dev)[:, zpad:]
    q = torch.empty(T, N, dtype=torch.int8, device=dev)
    s = torch.empty(T, N // 64, dtype=torch.float32, device=dev)
    out = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
    pkg.norm_gated_quant(v.to(dev), zd, w.to(dev), q, s)
    pkg.norm_gated(v.to(dev), zd, w.to(dev), out)
    zb = bits(zw[:, zpad:])
    rq, rs = O.norm_gated_quant(bits(v), zb, bits(w))
    assert_quant_close(q.cpu().numpy(), s.cpu().numpy(), rq, rs, f"norm_gated_quant T={T} HD={HD}")
    assert_bf16_close(bits(out), O.norm_gated(bits(v), zb, bits(w)), f"norm_gated T={T} HD={HD}")


@pytest.mark.parametrize("i", ["0", "1"])
def test_norm_gated_vs_reference_golden(pkg, dev, i):
    """The golden codes were made with bf16 truncation (CPU interpreter); the
    GPU rounds to nearest even, so compare with the oracle in that mode and
    check the oracle's trunc mode against the golden exactly."""
    p = f"norm_gated_{i}_"
    v, z, w = GOLD[p + "v"], GOLD[p + "z"], GOLD[p + "w"]
    T, N = v.shape
    q = torch.empty(T, N, dtype=torch.int8, device=dev)
    s = torch.empty(T, N // 64, dtype=torch.float32, device=dev)
    pkg.norm_gated_quant(bf16_t(v, dev), bf16_t(z, dev), bf16_t(w, dev), q, s)
    np.testing.assert_array_equal(O.norm_gated_quant(v, z, w, mode="trunc")[0], GOLD[p + "q"])
    rq, rs = O.norm_gated_quant(v, z, w)
    assert_quant_close(q.cpu().numpy(), s.cpu().numpy(), rq, rs, f"norm_gated golden {i}")


# ---------------------------------------------------------------- gate_mul_quant / silu_mul_quant
@pytest.mark.parametrize("M,NQ,HD,extra", [(1, 8, 256, 0), (4, 8, 256, 2048), (70, 8, 256, 64), (3, 2, 128, 0)])
def test_gate_mul_quant_vs_oracle(pkg, dev, M, NQ, HD, extra):
    g = torch.Generator().manual_seed(1300 + M + HD)
    N = NQ * HD
    a = rand_bf16(g, (M, N))
    proj = rand_bf16(g, (M, 2 * N + extra), 2.0)
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    s = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.gate_mul_quant(a.to(dev), proj.to(dev), q, s, hd=HD)
    y = O.gate_mul_y(bits(a), bits(proj), HD)
    assert_codes_near_ties(q.cpu().numpy(), s.cpu().numpy(), y, f"gate_mul_quant M={M}")


@pytest.mark.parametrize("i", ["0", "1"])
def test_gate_mul_quant_vs_reference_golden(pkg, dev, i):
    p = f"gate_mul_quant_{i}_"
    a, gt, hd = GOLD[p + "a"], GOLD[p + "g"], int(GOLD[p + "hd"])
    M, N = a.shape
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    s = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.gate_mul_quant(bf16_t(a, dev), bf16_t(gt, dev), q, s, hd=hd)
    assert_codes_near_ties(q.cpu().numpy(), s.cpu().numpy(), O.gate_mul_y(a, gt, hd), f"gate_mul golden {i}")


@pytest.mark.parametrize("M,N", [(1, 6144), (4, 512), (130, 2048)])
def test_silu_mul_quant_vs_oracle(pkg, dev, M, N):
    g = torch.Generator().manual_seed(1400 + M)
    gg = rand_bf16(g, (M, N), 2.0)
    uu = rand_bf16(g, (M, N))
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    s = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.silu_mul_quant(gg.to(dev), uu.to(dev), q, s)
    y = (O.silu(O.bf16_bits_to_f32(bits(gg))) * O.bf16_bits_to_f32(bits(uu))).astype(np.float32)
    assert_codes_near_ties(q.cpu().numpy(), s.cpu().numpy(), y, f"silu_mul_quant M={M}")


# ---------------------------------------------------------------- gate_proj
def _gate_proj_check(beta, gate, rb, rg, what):
    for got, ref, nm in ((beta, rb, "beta"), (gate, rg, "gate")):
        err = np.abs(got - ref)
        bad = err > 1e-5 + 1e-4 * np.abs(ref)
        assert not bad.any(), f"{what} {nm}: {int(bad.sum())} outside the bar, max err {err.max()}"


@pytest.mark.parametrize("M,K,NB", [(1, 2048, 16), (4, 2048, 16), (64, 1024, 16), (3, 2048, 32), (2, 320, 5)])
def test_gate_proj_vs_oracle(pkg, dev, M, K, NB):
    g = torch.Generator().manual_seed(1500 + M + NB)
    a = torch.randint(-127, 127, (M, K), dtype=torch.int8, generator=g)
    a_s = torch.rand(M, K // 64, generator=g) * 0.02
    wb, wa = rand_bf16(g, (NB, K), 0.05), rand_bf16(g, (NB, K), 0.05)
    dt, al = rand_bf16(g, (NB,)), rand_bf16(g, (NB,))
    beta = torch.empty(M, NB, device=dev)
    gate = torch.empty(M, NB, device=dev)
    rb_, rg_ = pkg.gate_proj(a.to(dev), a_s.to(dev), wb.to(dev), wa.to(dev), beta, gate, dt.to(dev), al.to(dev))
    assert rb_ is beta and rg_ is gate
    rb, rg = O.gate_proj(a.numpy(), a_s.numpy(), bits(wb), bits(wa), bits(dt), bits(al))
    _gate_proj_check(beta.cpu().numpy(), gate.cpu().numpy(), rb, rg, f"gate_proj M={M} K={K}")


@pytest.mark.parametrize("i", ["0", "1"])
def test_gate_proj_vs_reference_golden(pkg, dev, i):
    p = f"gate_proj_{i}_"
    a, a_s = GOLD[p + "a"], GOLD[p + "as"]
    M, K = a.shape
    NB = GOLD[p + "wb"].shape[0]
    beta = torch.empty(M, NB, device=dev)
    gate = torch.empty(M, NB, device=dev)
    pkg.gate_proj(torch.from_numpy(a).to(dev), torch.from_numpy(a_s).to(dev), bf16_t(GOLD[p + "wb"], dev),
                  bf16_t(GOLD[p + "wa"], dev), beta, gate, bf16_t(GOLD[p + "dt"], dev), bf16_t(GOLD[p + "alog"], dev))
    _gate_proj_check(beta.cpu().numpy(), gate.cpu().numpy(), GOLD[p + "beta"], GOLD[p + "gate"], f"golden {i}")


# ---------------------------------------------------------------- chains and errors
def test_rmsnorm_quant_feeds_gemm_under_graph(pkg, dev):
    """The engine's pattern: rmsnorm_quant then a projection of its codes,
    captured in a CUDA graph and replayed after refilling x in place."""
    g = torch.Generator().manual_seed(1600)
    M, K, N = 4, 2048, 1024
    w = rand_bf16(g, (K,), 0.2)
    b = torch.randint(-127, 127, (K, N), dtype=torch.int8, generator=g)
    bs = torch.rand(N, generator=g) * 0.002
    xd = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    q = torch.empty(M, K, dtype=torch.int8, device=dev)
    s = torch.empty(M, K // 64, dtype=torch.float32, device=dev)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    wd, bd, bsd = w.to(dev), b.to(dev), bs.to(dev)

    def step():
        pkg.rmsnorm_quant(xd, wd, q, s)
        pkg.gemm_i8(q, s, bd, bsd, out)
    side = torch.cuda.Stream(device=dev)
    xd.copy_(rand_bf16(g, (M, K)))
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()
    for _ in range(2):
        x = rand_bf16(g, (M, K))
        xd.copy_(x)
        graph.replay()
        torch.cuda.synchronize()
        y = O.rmsnorm_y(bits(x), bits(w))
        assert_codes_near_ties(q.cpu().numpy(), s.cpu().numpy(), y, "graph rmsnorm_quant")
        ref = O.gemm_i8(q.cpu().numpy(), s.cpu().numpy(), b.numpy(), bs.numpy())
        assert_bf16_close(bits(out), ref, "graph gemm after rmsnorm_quant")


def test_producer_shape_errors(pkg, dev):
    x = torch.zeros(2, 100, dtype=torch.bfloat16, device=dev)
    with pytest.raises(pkg._lib.QlinError):          # K not a multiple of 64 (C ABI)
        pkg.rmsnorm_quant(x, torch.zeros(100, dtype=torch.bfloat16, device=dev),
                          torch.empty(2, 100, dtype=torch.int8, device=dev),
                          torch.empty(2, 1, dtype=torch.float32, device=dev))
    with pytest.raises(ValueError):                  # w of the wrong length (binding)
        pkg.rmsnorm_quant(torch.zeros(2, 128, dtype=torch.bfloat16, device=dev),
                          torch.zeros(64, dtype=torch.bfloat16, device=dev),
                          torch.empty(2, 128, dtype=torch.int8, device=dev),
                          torch.empty(2, 2, dtype=torch.float32, device=dev))
    with pytest.raises(TypeError):                   # fp32 activations (binding)
        pkg.silu_mul_quant(torch.zeros(2, 64, device=dev), torch.zeros(2, 64, device=dev),
                           torch.empty(2, 64, dtype=torch.int8, device=dev),
                           torch.empty(2, 1, dtype=torch.float32, device=dev))
