"""Properties of the oracle's building blocks that the reference defines."""
import numpy as np

from oracle import qlin_oracle as O


def test_round_i8_half_away_and_clamp():
    v = np.array([0.5, -0.5, 1.5, -1.5, 2.5, 126.6, 127.4, 200.0, -200.0, 0.49999997, -0.49999997, 0.0],
                 dtype=np.float32)
    # kernels/common.py:24-29: trunc(v +- 0.5) in fp32, clamp +-127.  0.49999997 + 0.5
    # rounds to 1.0 in fp32, so it maps to 1 (not 0).
    assert O.round_i8(v).tolist() == [1, -1, 2, -2, 3, 127, 127, 127, -127, 1, -1, 0]


def test_bf16_rne_vs_trunc():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, -1.0 - 3 * 2 ** -9, 1.0 + 2 ** -9], dtype=np.float32)
    rne = O.bf16_bits_to_f32(O.f32_to_bf16_bits(x, "rne"))
    tr = O.bf16_bits_to_f32(O.f32_to_bf16_bits(x, "trunc"))
    assert rne.tolist() == [1.0, 1.0 + 2 ** -7, -1.0 - 2 ** -7, 1.0]
    assert tr.tolist() == [1.0, 1.0, -1.0, 1.0]


def test_unpack_w4_layout():
    # byte j of column n: k=2j low nibble, k=2j+1 high nibble (kernels/w4.py:3-15)
    b = np.array([[0x21, 0xF0]], dtype=np.uint8)           # K=2, N=2
    w = O.unpack_w4(b, None, 2)
    assert w.tolist() == [[1 - 8, 0 - 8], [2 - 8, 15 - 8]]
    z = np.array([[3, 15]], dtype=np.uint8)
    w = O.unpack_w4(b, z, 2)
    assert w.tolist() == [[1 - 3, 0 - 15], [2 - 3, 15 - 15]]


def test_quant_groups_zero_group_scale_floor():
    y = np.zeros((1, 64), dtype=np.float32)
    q, s = O.quant_groups(y)
    assert (q == 0).all() and s[0, 0] == np.float32(1e-8)


def test_w4_sub_block():
    assert O.w4_sub(32) == 32 and O.w4_sub(64) == 64 and O.w4_sub(128) == 64


def test_gemm_linear_in_weight_scale():
    """out * 2 == gemm with b_s * 2 (exact: power-of-two scaling)."""
    rng = np.random.default_rng(0)
    a = rng.integers(-127, 127, (3, 128), dtype=np.int8)
    s = rng.random((3, 2), dtype=np.float32) * 0.02
    b = rng.integers(-127, 127, (128, 32), dtype=np.int8)
    bs = rng.random(32, dtype=np.float32) * 0.002
    o1 = O.gemm_i8_f32(a, s, b, bs)
    o2 = O.gemm_i8_f32(a, s, b, (bs * 2).astype(np.float32))
    np.testing.assert_array_equal(o1 * 2, o2)
