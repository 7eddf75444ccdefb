"""GPU parity of the large-M (prefill) tensor-core GEMM path against the CPU oracle.

W8 projections with M >= 128 rows take the tcgen05 GEMM (128-row x 256-column
tiles, per-64-K-group int32 promoted with the activation row scale).  Same
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
