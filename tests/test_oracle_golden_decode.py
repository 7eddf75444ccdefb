"""The CPU oracle's decode-step neighbours reproduce the reference's own
outputs bit for bit.

Fixtures in tests/golden/ref_golden_decode.npz come from running the
reference's kernels/attention.py and kernels/linear_attn.py under the Triton
CPU interpreter (tests/golden/make_golden.py ... decode).  The interpreter
truncates fp32 -> bf16, so every bf16 output is compared with the oracle in
its mode="trunc"; int8 KV codes, their scales and the fp32 recurrent state
involve no bf16 rounding.
"""
import os

import numpy as np
import pytest

from oracle import qlin_oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden_decode.npz"))
NQ, NKV, HD = 8, 2, 256


def _cases(prefix):
    ids = {k[len(prefix):].split("_")[0] for k in GOLD.files if k.startswith(prefix)}
    return sorted(i for i in ids if i.isdigit())


@pytest.mark.parametrize("i", _cases("qk_rope_"))
def test_qk_norm_rope(i):
    p = f"qk_rope_{i}_"
    T, pos0, int8, batch, seq = (int(v) for v in GOLD[p + "cfg"])
    rows = T * seq if batch else seq
    if int8:
        kvc = np.zeros((rows, 2 * NKV * HD), dtype=np.int8)
        kvs = np.zeros((rows, 2 * NKV), dtype=np.float32)
    else:
        kvc = np.zeros((rows, 2 * NKV * HD), dtype=np.uint16)
        kvs = None
    q = O.qk_norm_rope(GOLD[p + "proj"], GOLD[p + "qn"], GOLD[p + "kn"], GOLD[p + "invf"], NQ, NKV, HD, pos0, kvc,
                       kvs, batch=bool(batch), mode="trunc")
    np.testing.assert_array_equal(q, GOLD[p + "q"])
    np.testing.assert_array_equal(kvc, GOLD[p + "kvc"])
    if int8:
        np.testing.assert_array_equal(kvs.view(np.uint32), GOLD[p + "kvs"].view(np.uint32))


@pytest.mark.parametrize("i", _cases("attn_decode_"))
def test_attn_decode(i):
    p = f"attn_decode_{i}_"
    B, pos, int8 = (int(v) for v in GOLD[p + "cfg"])
    out = O.attn_decode(GOLD[p + "q"], GOLD[p + "kvc"], pos, GOLD[p + "kvs"] if int8 else None, batch=B,
                        mode="trunc")
    np.testing.assert_array_equal(out, GOLD[p + "out"])


@pytest.mark.parametrize("i", _cases("delta_decode_"))
def test_delta_decode(i):
    p = f"delta_decode_{i}_"
    state = GOLD[p + "state"].copy()
    out = O.delta_decode(GOLD[p + "qkv"], GOLD[p + "g"], GOLD[p + "beta"], state, mode="trunc")
    np.testing.assert_array_equal(out, GOLD[p + "out"])
    np.testing.assert_array_equal(state[:2].view(np.uint32), GOLD[p + "state_out2"].view(np.uint32))


@pytest.mark.parametrize("i", _cases("conv_"))
def test_conv(i):
    p = f"conv_{i}_"
    T, batch = (int(v) for v in GOLD[p + "cfg"])
    y = O.conv_silu(GOLD[p + "x"], GOLD[p + "w"], GOLD[p + "state"], T, batch=bool(batch), mode="trunc")
    np.testing.assert_array_equal(y, GOLD[p + "y"])
    st = O.conv_state_update(GOLD[p + "x"], GOLD[p + "state"], T, batch=T if batch else 1)
    np.testing.assert_array_equal(st, GOLD[p + "state_out"])


@pytest.mark.parametrize("i", _cases("attn_prefill_"))
def test_attn_prefill(i):
    p = f"attn_prefill_{i}_"
    T, pos0, int8 = (int(v) for v in GOLD[p + "cfg"])
    out = O.attn_prefill(GOLD[p + "q"], GOLD[p + "kvc"], T, pos0, GOLD[p + "kvs"] if int8 else None, mode="trunc")
    np.testing.assert_array_equal(out, GOLD[p + "out"])


@pytest.mark.parametrize("i", _cases("delta_prefill_"))
def test_delta_prefill(i):
    p = f"delta_prefill_{i}_"
    state = GOLD[p + "state"].copy()
    T = GOLD[p + "qkv"].shape[0]
    out = O.delta_prefill(GOLD[p + "qkv"], GOLD[p + "g"], GOLD[p + "beta"], state, T, mode="trunc")
    np.testing.assert_array_equal(out, GOLD[p + "out"])
    np.testing.assert_array_equal(state[:2].view(np.uint32), GOLD[p + "state_out2"].view(np.uint32))
