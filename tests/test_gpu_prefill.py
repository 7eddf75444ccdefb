"""GPU parity of the large-M (prefill) tensor-core GEMM paths against the CPU oracle.

W8 projections and W4 projections (weight groups of 64 * k) with M >= 128
rows take the tcgen05 GEMMs (128-row x 256-column tiles, per-64-K-group int32
promoted with the activation row scale, times the group weight scale for W4).  Same
bars as the small-M tests: bf16 within 1e-3 + 1e-2|ref|, integer work bit
exact (unit scales), untouched columns outside the output stay untouched.
Config 3 (M = 2048, K = 2048, N = 12288) is checked on the full output for
finite values and on sampled rows against the oracle (rows are independent).
"""
import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O
from qlin_testutil import acts_ref, acts_x, assert_bf16_close, bits, gen, w8

pytestmark = pytest.mark.gpu


def cu(t):
    return None if t is None else t.to("cuda:0")


@pytest.mark.parametrize("M", [128, 129, 200, 256, 300])
@pytest.mark.parametrize("N,K", [(144, 64), (272, 192), (400, 1024), (2048, 2048)])
def test_prefill_gemm_i8_residual_alias(pkg, dev, M, N, K):
    g = gen(6000 + M * 3 + N + K)
    a, s = acts_ref(g, M, K)
    b, bs = w8(g, K, N)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    buf = torch.zeros(M, N + 16, dtype=torch.bfloat16, device=dev)
    out = buf[:, 8:8 + N]
    out.copy_(res.to(dev))
    pkg.gemm_i8(cu(a), cu(s), cu(b), cu(bs), out, residual=out)
    ref = O.gemm_i8(a.numpy(), s.numpy(), b.numpy(), bs.numpy(), bits(res))
    assert_bf16_close(bits(out), ref, f"prefill gemm_i8 M={M} N={N} K={K}")
    assert (bits(buf[:, :8]) == 0).all() and (bits(buf[:, 8 + N:]) == 0).all()


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (257, 1024, 512), (512, 384, 2048)])
def test_prefill_integer_exact(pkg, dev, M, N, K):
    """Unit scales: every fp32 step is exact, so the bf16 output must equal the
    exact integer product bit for bit (the promotion through the 2^23 + 2^22
    bit pattern recovers each group's int32 sum exactly)."""
    g = gen(6100 + M + N)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, generator=g)
    b = torch.randint(-128, 128, (K, N), dtype=torch.int8, generator=g)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    pkg.gemm_i8(cu(a), cu(torch.ones(M, K // 64)), cu(b), cu(torch.ones(N)), out)
    exact = a.double() @ b.double()
    np.testing.assert_array_equal(bits(out), O.f32_to_bf16_bits(exact.numpy().astype(np.float32)))


@pytest.mark.parametrize("M", [128, 300])
def test_prefill_proj3(pkg, dev, M):
    K = 2048
    g = gen(6200 + M)
    a, s = acts_x(g, M, K)
    ns = (4096, 512, 528)
    ws = [w8(g, K, n, "lognormal") for n in ns]
    out = torch.zeros(M, sum(ns) + 256, dtype=torch.bfloat16, device=dev)
    pkg.proj3(cu(a), cu(s), cu(ws[0][0]), cu(ws[0][1]), cu(ws[1][0]), cu(ws[1][1]), cu(ws[2][0]),
              cu(ws[2][1]), out)
    ref = O.proj3(a.numpy(), s.numpy(), [(w.numpy(), sc.numpy(), None) for w, sc in ws])
    assert_bf16_close(bits(out)[:, :sum(ns)], ref, f"prefill proj3 M={M}")
    assert (bits(out)[:, sum(ns):] == 0).all()


def test_prefill_unaligned_row_stride(pkg, dev):
    """Row strides that rule out 16-byte vector stores take the scalar path."""
    M, N, K = 160, 256, 256
    g = gen(6300)
    a, s = acts_ref(g, M, K)
    b, bs = w8(g, K, N)
    res_buf = torch.randn(M, N + 3, generator=g).to(torch.bfloat16)
    buf = torch.zeros(M, N + 5, dtype=torch.bfloat16, device=dev)
    out = buf[:, 1:1 + N]
    pkg.gemm_i8(cu(a), cu(s), cu(b), cu(bs), out, residual=cu(res_buf)[:, :N])
    ref = O.gemm_i8(a.numpy(), s.numpy(), b.numpy(), bs.numpy(), bits(res_buf[:, :N]))
    assert_bf16_close(bits(out), ref, "prefill unaligned strides")
    assert (bits(buf[:, :1]) == 0).all() and (bits(buf[:, 1 + N:]) == 0).all()


@pytest.mark.parametrize("M", [512, 2048])
def test_config3_prefill_w8a8(pkg, dev, M):
    """Config 3: X ~ N(0,1) with 0.1 % outliers x20, quantised on the GPU by
    quant_row (bit-exact with the oracle), then the W8A8 GEMM against W int8
    [2048, 12288] with lognormal(-6, 0.5) scales; 64 sampled rows checked
    against the oracle, every output finite."""
    K, N = 2048, 12288
    g = gen(6400 + M)
    x = torch.randn(M, K, generator=g)
    x[torch.rand(M, K, generator=g) < 0.001] *= 20.0
    xb = x.to(torch.bfloat16)
    q = torch.empty(M, K, dtype=torch.int8, device=dev)
    s = torch.empty(M, K // 64, dtype=torch.float32, device=dev)
    pkg.quant_row(cu(xb), q, s)
    rq, rs = O.quant_row(bits(xb))
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    b, bs = w8(g, K, N, "lognormal")
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    pkg.gemm_i8(q, s, cu(b), cu(bs), out)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    rows = np.sort(np.random.default_rng(M).choice(M, 64, replace=False))
    ref = O.gemm_i8(rq[rows], rs[rows], b.numpy(), bs.numpy())
    assert_bf16_close(bits(out)[rows], ref, f"config 3 M={M}")


def test_prefill_matches_small_m_path_at_threshold(pkg, dev):
    """Row 127 goes through the small-M kernel, 128 through the GEMM: both
    within tolerance of the oracle on the same data."""
    K, N = 1024, 512
    g = gen(6500)
    a, s = acts_x(g, 128, K)
    b, bs = w8(g, K, N, "lognormal")
    ref = O.gemm_i8(a.numpy(), s.numpy(), b.numpy(), bs.numpy())
    for M in (127, 128):
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        pkg.gemm_i8(cu(a[:M]), cu(s[:M]), cu(b), cu(bs), out)
        assert_bf16_close(bits(out), ref[:M], f"threshold M={M}")


# ----------------------------------------------------------------------------- W4 (groups of 64 * k)
from qlin_testutil import w4  # noqa: E402


@pytest.mark.parametrize("M", [128, 200, 300])
@pytest.mark.parametrize("wg,zeros", [(64, True), (128, True), (128, False), (256, True), (192, True)])
def test_prefill_gemm_w4(pkg, dev, M, wg, zeros):
    K = 768 if wg == 192 else 1024
    N = 400
    g = gen(6600 + M + wg + zeros)
    a, s = acts_x(g, M, K)
    b, sc, z = w4(g, K, N, wg, zeros)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    out = res.clone().to(dev)
    pkg.gemm_w4(cu(a), cu(s), cu(b), cu(sc), out, residual=out, b_z=cu(z))
    ref = O.gemm_w4(a.numpy(), s.numpy(), b.numpy(), bits(sc), None if z is None else z.numpy(), bits(res))
    assert_bf16_close(bits(out), ref, f"prefill gemm_w4 M={M} wg={wg} zeros={zeros}")


@pytest.mark.parametrize("M,K,wg", [(128, 192, 64), (256, 2048, 128)])
def test_prefill_w4_integer_exact(pkg, dev, M, K, wg):
    """Unit scales: the output is the exact integer sum of a * (nibble - z)."""
    N = 272
    g = gen(6700 + M)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g)
    b, _, z = w4(g, K, N, wg, True)
    sc = torch.ones(K // wg, N, dtype=torch.bfloat16)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    pkg.gemm_w4(cu(a), cu(torch.ones(M, K // 64)), cu(b), cu(sc), out, b_z=cu(z))
    w = O.unpack_w4(b.numpy(), z.numpy(), wg).astype(np.float64)
    exact = a.numpy().astype(np.float64) @ w
    np.testing.assert_array_equal(bits(out), O.f32_to_bf16_bits(exact.astype(np.float32)))


@pytest.mark.parametrize("M,K,N", [(256, 4096, 640), (128, 8192, 640), (64, 8192, 1280)])
def test_prefill_w4_k_parts_integer_exact(pkg, dev, M, K, N):
    """Few output tiles (a column shard of a tensor-parallel down projection):
    each tile's K is cut into parts on several CTAs (14, 16 and 14 parts here,
    rows shared unevenly among them) whose sums meet in a workspace; M = 64
    takes this GEMM through the long-K mid-M rule.  Unit scales: every part's
    fp32 sum and their total are exact integers."""
    g = gen(6750 + M)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g)
    b, _, z = w4(g, K, N, 128, True)
    sc = torch.ones(K // 128, N, dtype=torch.bfloat16)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    pkg.gemm_w4(cu(a), cu(torch.ones(M, K // 64)), cu(b), cu(sc), out, b_z=cu(z))
    w = O.unpack_w4(b.numpy(), z.numpy(), 128).astype(np.float64)
    exact = a.numpy().astype(np.float64) @ w
    np.testing.assert_array_equal(bits(out), O.f32_to_bf16_bits(exact.astype(np.float32)))


def test_prefill_proj3_w4(pkg, dev):
    M, K, wg = 160, 2048, 128
    g = gen(6800)
    a, s = acts_x(g, M, K)
    s1 = w4(g, K, 2048, wg, True)
    s2 = w4(g, K, 528, wg, True)
    out = torch.zeros(M, 2576 + 128, dtype=torch.bfloat16, device=dev)
    pkg.proj3_w4(cu(a), cu(s), cu(s1[0]), cu(s1[1]), cu(s2[0]), cu(s2[1]), None, None, out,
                 z1=cu(s1[2]), z2=cu(s2[2]))
    ref = O.proj3(a.numpy(), s.numpy(), [(s1[0].numpy(), bits(s1[1]), s1[2].numpy()),
                                         (s2[0].numpy(), bits(s2[1]), s2[2].numpy())])
    assert_bf16_close(bits(out)[:, :2576], ref, "prefill proj3_w4")
    assert (bits(out)[:, 2576:] == 0).all()


def test_config3_prefill_w4_variant(pkg, dev):
    """Config 3's W4 variant: M = 2048, K = 2048, N = 12288, group 128 with zeros;
    64 sampled rows against the oracle, every output finite."""
    M, K, N, wg = 2048, 2048, 12288, 128
    g = gen(6900)
    a, s = acts_x(g, M, K, outliers=True)
    b, sc, z = w4(g, K, N, wg, True)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    pkg.gemm_w4(cu(a), cu(s), cu(b), cu(sc), out, b_z=cu(z))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    rows = np.sort(np.random.default_rng(7).choice(M, 64, replace=False))
    ref = O.gemm_w4(a.numpy()[rows], s.numpy()[rows], b.numpy(), bits(sc), z.numpy())
    assert_bf16_close(bits(out)[rows], ref, "config 3 W4")


# ----------------------------------------------------------------------------- fused gate/up at M >= 128
from qlin_testutil import assert_quant_close  # noqa: E402


@pytest.mark.parametrize("M,K,N", [(128, 1024, 384), (300, 2048, 1024)])
def test_prefill_gate_up_quant_w8(pkg, dev, M, K, N):
    g = gen(7100 + M)
    a, s = acts_x(g, M, K)
    wg, sg = w8(g, K, N, "lognormal")
    wu, su = w8(g, K, N, "lognormal")
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    qs = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.mlp_gate_up_quant(cu(a), cu(s), cu(wg), cu(sg), cu(wu), cu(su), q, qs)
    rq, rs = O.mlp_gate_up_quant(a.numpy(), s.numpy(), wg.numpy(), sg.numpy(), wu.numpy(), su.numpy())
    assert_quant_close(q.cpu().numpy(), qs.cpu().numpy(), rq, rs, f"prefill gate_up_quant W8 M={M}")


@pytest.mark.parametrize("M,N", [(128, 400), (257, 512)])
def test_prefill_gate_up_bf16_w8(pkg, dev, M, N):
    K = 1024
    g = gen(7200 + M)
    a, s = acts_x(g, M, K)
    wg, sg = w8(g, K, N, "lognormal")
    wu, su = w8(g, K, N, "lognormal")
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    pkg.mlp_gate_up(cu(a), cu(s), cu(wg), cu(sg), cu(wu), cu(su), out)
    ref = O.mlp_gate_up(a.numpy(), s.numpy(), wg.numpy(), sg.numpy(), wu.numpy(), su.numpy())
    assert_bf16_close(bits(out), ref, f"prefill gate_up bf16 M={M} N={N}")


@pytest.mark.parametrize("M,wg,zeros", [(128, 128, True), (300, 64, False), (200, 256, True)])
def test_prefill_gate_up_quant_w4(pkg, dev, M, wg, zeros):
    K, N = 1024, 512
    g = gen(7300 + M + wg)
    a, s = acts_x(g, M, K)
    gw, gs, gz = w4(g, K, N, wg, zeros)
    uw, us, uz = w4(g, K, N, wg, zeros)
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    qs = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.mlp_gate_up_quant_w4(cu(a), cu(s), cu(gw), cu(gs), cu(uw), cu(us), q, qs, zg=cu(gz), zu=cu(uz))
    rq, rs = O.mlp_gate_up_quant_w4(a.numpy(), s.numpy(), gw.numpy(), bits(gs), uw.numpy(), bits(us),
                                    None if gz is None else gz.numpy(), None if uz is None else uz.numpy())
    assert_quant_close(q.cpu().numpy(), qs.cpu().numpy(), rq, rs, f"prefill gate_up_quant W4 M={M} wg={wg}")


def test_prefill_gate_up_quant_w4_k_parts(pkg, dev):
    """A column shard of the config-5 gate/up (5 tiles of 128 gate + 128 up
    columns at M = 256): K parts on several CTAs per tile, then the fused
    SiLU + requantisation on the summed parts."""
    M, K, N = 256, 2048, 640
    g = gen(7350)
    a, s = acts_x(g, M, K)
    gw, gs, gz = w4(g, K, N, 128, True)
    uw, us, uz = w4(g, K, N, 128, True)
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    qs = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.mlp_gate_up_quant_w4(cu(a), cu(s), cu(gw), cu(gs), cu(uw), cu(us), q, qs, zg=cu(gz), zu=cu(uz))
    rq, rs = O.mlp_gate_up_quant_w4(a.numpy(), s.numpy(), gw.numpy(), bits(gs), uw.numpy(), bits(us),
                                    gz.numpy(), uz.numpy())
    assert_quant_close(q.cpu().numpy(), qs.cpu().numpy(), rq, rs, "prefill gate_up_quant W4 K parts")


# ----------------------------------------------------------------------------- mid M (33..127), many tiles
# Below 128 rows, shapes with at least 64 GEMM tiles take the tensor-core GEMM
# (one pass over the weights) instead of small-M row blocks.
@pytest.mark.parametrize("M,N,K", [(33, 16384, 256), (64, 16384, 512), (100, 16512, 256)])
def test_mid_m_gemm_i8_many_tiles(pkg, dev, M, N, K):
    g = gen(8100 + M)
    a, s = acts_ref(g, M, K)
    b, bs = w8(g, K, N)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    out = res.clone().to(dev)
    pkg.gemm_i8(cu(a), cu(s), cu(b), cu(bs), out, residual=out)
    ref = O.gemm_i8(a.numpy(), s.numpy(), b.numpy(), bs.numpy(), bits(res))
    assert_bf16_close(bits(out), ref, f"mid-M gemm_i8 M={M} N={N}")


@pytest.mark.parametrize("M,wg,zeros", [(40, 128, True), (64, 64, False), (127, 128, True)])
def test_mid_m_gemm_w4_many_tiles(pkg, dev, M, wg, zeros):
    K, N = 512, 16384
    g = gen(8200 + M + wg)
    a, s = acts_x(g, M, K)
    b, sc, z = w4(g, K, N, wg, zeros)
    out = torch.zeros(M, N, dtype=torch.bfloat16, device=dev)
    pkg.gemm_w4(cu(a), cu(s), cu(b), cu(sc), out, b_z=cu(z))
    ref = O.gemm_w4(a.numpy(), s.numpy(), b.numpy(), bits(sc), None if z is None else z.numpy())
    assert_bf16_close(bits(out), ref, f"mid-M gemm_w4 M={M} wg={wg}")


@pytest.mark.parametrize("M", [48, 100])
def test_mid_m_gate_up_quant_w4_many_tiles(pkg, dev, M):
    K, N, wg = 256, 8192, 128
    g = gen(8300 + M)
    a, s = acts_x(g, M, K)
    gw, gs, gz = w4(g, K, N, wg, True)
    uw, us, uz = w4(g, K, N, wg, True)
    q = torch.empty(M, N, dtype=torch.int8, device=dev)
    qs = torch.empty(M, N // 64, dtype=torch.float32, device=dev)
    pkg.mlp_gate_up_quant_w4(cu(a), cu(s), cu(gw), cu(gs), cu(uw), cu(us), q, qs, zg=cu(gz), zu=cu(uz))
    rq, rs = O.mlp_gate_up_quant_w4(a.numpy(), s.numpy(), gw.numpy(), bits(gs), uw.numpy(), bits(us),
                                    gz.numpy(), uz.numpy())
    assert_quant_close(q.cpu().numpy(), qs.cpu().numpy(), rq, rs, f"mid-M gate_up_quant W4 M={M}")
