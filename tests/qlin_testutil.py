"""Shared helpers for the parity tests: seeded generators for the engine
layouts, bf16 bit conversions and the tolerance checks."""
import numpy as np
import torch

from oracle import qlin_oracle as O

GROUP = 64
# bf16 outputs: |ours - oracle| <= ATOL + RTOL * |oracle| elementwise
ATOL = 1e-3
RTOL = 1e-2


def bits(t):
    """bf16 tensor (any device) -> uint16 numpy bit pattern."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def assert_bf16_close(got_bits, ref_bits, what=""):
    got = O.bf16_bits_to_f32(got_bits)
    ref = O.bf16_bits_to_f32(ref_bits)
    err = np.abs(got - ref)
    bound = ATOL + RTOL * np.abs(ref)
    bad = ~(err <= bound)
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} outside |d| <= {ATOL} + {RTOL}|ref|; first at "
            f"{tuple(i)}: got {got[tuple(i)]} ref {ref[tuple(i)]}")


def assert_quant_close(q, s, rq, rs, what=""):
    """Fused quantisation outputs: >= 99.9 % of int8 codes equal, all within +-1,
    scales within 1e-2 relative (silu's exp differs in ulps between
    implementations; kernels/gemm.py:198-211 rounds h through bf16 first)."""
    d = q.astype(np.int32) - rq.astype(np.int32)
    eq = float((d == 0).mean())
    assert np.abs(d).max() <= 1, f"{what}: int8 code differs by {np.abs(d).max()}"
    assert eq >= 0.999, f"{what}: only {eq * 100:.3f}% int8 codes equal"
    np.testing.assert_allclose(s, rs, rtol=1e-2, atol=0, err_msg=what)


def gen(seed):
    return torch.Generator().manual_seed(seed)


def acts_ref(g, M, K):
    """.dev/test_kernels.py:34-36 distributions."""
    a = torch.randint(-127, 127, (M, K), dtype=torch.int8, generator=g)
    s = torch.rand(M, K // GROUP, generator=g) * 0.02
    return a, s


def acts_x(g, M, K, outliers=False):
    """bf16 X ~ N(0,1) (optionally 0.1 % entries x20) quantised by the oracle's quant_row."""
    x = torch.randn(M, K, generator=g)
    if outliers:
        x[torch.rand(M, K, generator=g) < 0.001] *= 20.0
    xb = x.to(torch.bfloat16)
    q, s = O.quant_row(bits(xb))
    return torch.from_numpy(q), torch.from_numpy(s)


def w8(g, K, N, dist="ref"):
    b = torch.randint(-127, 127, (K, N), dtype=torch.int8, generator=g)
    if dist == "ref":
        bs = torch.rand(N, generator=g) * 0.002
    else:   # lognormal(-6, 0.5)
        bs = torch.exp(torch.randn(N, generator=g) * 0.5 - 6.0)
    return b, bs


def w4(g, K, N, wg, zeros):
    b = torch.randint(0, 256, (K // 2, N), dtype=torch.int32, generator=g).to(torch.uint8)
    s = torch.exp(torch.randn(K // wg, N, generator=g) * 0.5 - 5.0).to(torch.bfloat16)
    z = torch.randint(0, 16, (K // wg, N), dtype=torch.int32, generator=g).to(torch.uint8) if zeros else None
    return b, s, z
