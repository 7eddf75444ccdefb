"""The CPU oracle reproduces the reference's own outputs bit for bit.

Fixtures in tests/golden/ref_golden.npz were produced by running the
reference's Triton kernels under the Triton CPU interpreter
(tests/golden/make_golden.py).  The interpreter truncates fp32 -> bf16, so the
oracle runs in mode="trunc" here; everything else is the same code path the
GPU parity tests use with round-to-nearest-even.
"""
import os

import numpy as np
import pytest

from oracle import qlin_oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz"))


def _get(p, k):
    return GOLD[p + k] if (p + k) in GOLD.files else None


def _cases(prefix):
    ids = {k[len(prefix):].split("_")[0] for k in GOLD.files if k.startswith(prefix)}
    return sorted(i for i in ids if i.isdigit())


@pytest.mark.parametrize("i", _cases("quant_row_"))
def test_quant_row(i):
    p = f"quant_row_{i}_"
    q, s = O.quant_row(GOLD[p + "x"])
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    np.testing.assert_array_equal(s.view(np.uint32), GOLD[p + "s"].view(np.uint32))


@pytest.mark.parametrize("i", _cases("gemm_i8_"))
def test_gemm_i8(i):
    p = f"gemm_i8_{i}_"
    out = O.gemm_i8(GOLD[p + "a"], GOLD[p + "as"], GOLD[p + "b"], GOLD[p + "bs"], _get(p, "res"),
                    mode="trunc")
    np.testing.assert_array_equal(out, GOLD[p + "out"])


@pytest.mark.parametrize("i", _cases("gemm_w4_"))
def test_gemm_w4(i):
    p = f"gemm_w4_{i}_"
    out = O.gemm_w4(GOLD[p + "a"], GOLD[p + "as"], GOLD[p + "b"], GOLD[p + "bs"], _get(p, "bz"),
                    _get(p, "res"), mode="trunc")
    np.testing.assert_array_equal(out, GOLD[p + "out"])


@pytest.mark.parametrize("prefix", ["proj3_0_", "proj3_1_", "proj3_w4_0_", "proj3_w4_1_"])
def test_proj3(prefix):
    segs = [(GOLD[prefix + f"w{j}"], GOLD[prefix + f"s{j}"], _get(prefix, f"z{j}"))
            if prefix + f"w{j}" in GOLD.files else None for j in range(3)]
    out = O.proj3(GOLD[prefix + "a"], GOLD[prefix + "as"], segs, mode="trunc")
    ref = GOLD[prefix + "out"]
    np.testing.assert_array_equal(out, ref[:, :out.shape[1]])
    assert (ref[:, out.shape[1]:] == 0).all()     # columns past N1+N2+N3 untouched


@pytest.mark.parametrize("i", _cases("gate_up_"))
def test_gate_up_w8(i):
    p = f"gate_up_{i}_"
    args = (GOLD[p + "a"], GOLD[p + "as"], GOLD[p + "wg"], GOLD[p + "sg"], GOLD[p + "wu"], GOLD[p + "su"])
    np.testing.assert_array_equal(O.mlp_gate_up(*args, mode="trunc"), GOLD[p + "h"])
    q, s = O.mlp_gate_up_quant(*args, mode="trunc")
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    np.testing.assert_array_equal(s.view(np.uint32), GOLD[p + "qs"].view(np.uint32))


@pytest.mark.parametrize("i", _cases("gate_up_w4_"))
def test_gate_up_w4(i):
    p = f"gate_up_w4_{i}_"
    q, s = O.mlp_gate_up_quant_w4(GOLD[p + "a"], GOLD[p + "as"], GOLD[p + "wg"], GOLD[p + "sg"],
                                  GOLD[p + "wu"], GOLD[p + "su"], _get(p, "zg"), _get(p, "zu"),
                                  mode="trunc")
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    np.testing.assert_array_equal(s.view(np.uint32), GOLD[p + "qs"].view(np.uint32))


def test_fixture_coverage():
    """Every hot-path entry point has golden vectors."""
    for prefix in ("quant_row_", "gemm_i8_", "gemm_w4_", "proj3_0_", "proj3_w4_", "gate_up_0_",
                   "gate_up_w4_"):
        assert any(k.startswith(prefix) for k in GOLD.files), prefix
