"""The CPU oracle's activation producers reproduce the reference's own
outputs bit for bit.

Fixtures in tests/golden/ref_golden_norm.npz come from running the
reference's kernels/norm.py under the Triton CPU interpreter
(tests/golden/make_golden.py ... norm).  The interpreter truncates fp32 ->
bf16, so the one producer that rounds through bf16 before quantising
(norm_gated_quant, and the bf16 output of norm_gated) is pinned in the
oracle's mode="trunc".
"""
import os

import numpy as np
import pytest

from oracle import qlin_oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden_norm.npz"))


def _cases(prefix):
    ids = {k[len(prefix):].split("_")[0] for k in GOLD.files if k.startswith(prefix)}
    return sorted(i for i in ids if i.isdigit())


def _same_f32(a, b):
    np.testing.assert_array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("i", _cases("rmsnorm_quant_"))
def test_rmsnorm_quant(i):
    p = f"rmsnorm_quant_{i}_"
    q, s = O.rmsnorm_quant(GOLD[p + "x"], GOLD[p + "w"], 1e-6, bool(GOLD[p + "one_plus"]))
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    _same_f32(s, GOLD[p + "s"])


@pytest.mark.parametrize("i", _cases("norm_gated_"))
def test_norm_gated(i):
    p = f"norm_gated_{i}_"
    q, s = O.norm_gated_quant(GOLD[p + "v"], GOLD[p + "z"], GOLD[p + "w"], 1e-6, mode="trunc")
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    _same_f32(s, GOLD[p + "s"])
    np.testing.assert_array_equal(O.norm_gated(GOLD[p + "v"], GOLD[p + "z"], GOLD[p + "w"], 1e-6, mode="trunc"),
                                  GOLD[p + "out"])


@pytest.mark.parametrize("i", _cases("gate_mul_quant_"))
def test_gate_mul_quant(i):
    p = f"gate_mul_quant_{i}_"
    q, s = O.gate_mul_quant(GOLD[p + "a"], GOLD[p + "g"], int(GOLD[p + "hd"]))
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    _same_f32(s, GOLD[p + "s"])


def test_silu_mul_quant():
    q, s = O.silu_mul_quant(GOLD["silu_mul_quant_0_g"], GOLD["silu_mul_quant_0_u"])
    np.testing.assert_array_equal(q, GOLD["silu_mul_quant_0_q"])
    _same_f32(s, GOLD["silu_mul_quant_0_s"])


@pytest.mark.parametrize("i", _cases("gate_proj_"))
def test_gate_proj(i):
    p = f"gate_proj_{i}_"
    beta, gate = O.gate_proj(GOLD[p + "a"], GOLD[p + "as"], GOLD[p + "wb"], GOLD[p + "wa"], GOLD[p + "dt"],
                             GOLD[p + "alog"])
    _same_f32(beta, GOLD[p + "beta"])
    _same_f32(gate, GOLD[p + "gate"])


def test_fixture_coverage():
    for prefix in ("rmsnorm_quant_", "norm_gated_", "gate_mul_quant_", "silu_mul_quant_", "gate_proj_"):
        assert any(k.startswith(prefix) for k in GOLD.files), prefix
