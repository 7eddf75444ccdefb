"""Decode-step neighbours (kernels/attention.py, kernels/linear_attn.py) on
the CUDA path against the CPU oracle and the reference's own outputs.

Parity rules:
* bf16 outputs (q after RoPE, bf16 K/V rows, attention output, delta-rule
  output, conv output): |d| <= 1e-3 + 1e-2 |ref| elementwise;
* int8 K/V codes: equal except where the oracle's value / scale lies within
  1e-4 of a .5 rounding boundary (trig and sums in another order move the
  last bits), where they may differ by one; their scales within 1e-5;
* the fp32 delta-rule state: |d| <= 1e-6 + 1e-5 |ref| (sums over DK in
  another order);
* the conv window update is a copy: bit-exact.
"""
import os

import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O
from qlin_testutil import assert_bf16_close, bits, from_bits

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden_decode.npz"))
NQ, NKV, HD, RD = 8, 2, 256, 64
NH, DK, DV = 16, 128, 128
CONV = 2 * NH * DK + NH * DV


def invf_t():
    return 1.0 / (1e7 ** (torch.arange(0, RD, 2, dtype=torch.float32) / RD))


def rand_bf16(g, shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def assert_kv_codes(codes, scales, ref_y, what):
    """codes int8 [n, hd], scales [n] from the GPU; ref_y fp32 [n, hd] the
    oracle's values before quantisation."""
    rq = np.empty_like(codes)
    rs = np.empty(ref_y.shape[0], dtype=np.float32)
    for i in range(ref_y.shape[0]):
        rq[i], rs[i] = O._quant_vec(ref_y[i])
    np.testing.assert_allclose(scales, rs, rtol=1e-5, atol=0, err_msg=f"{what}: scales")
    d = codes.astype(np.int32) - rq.astype(np.int32)
    v = np.abs(ref_y / rs[:, None])
    near = np.abs(v - np.floor(v) - 0.5) < 1e-4
    bad = (d != 0) & ~(near & (np.abs(d) == 1))
    assert not bad.any(), f"{what}: {int(bad.sum())} codes differ away from a rounding tie"


def oracle_kv(proj_bits, kn_bits, v_off, row, pos, head):
    """The oracle's fp32 K (head < NKV) or V vector of one cache row."""
    p = O.bf16_bits_to_f32(proj_bits)
    off = 2 * NQ * HD
    if head < NKV:
        return O._norm_rope(p[row, off + head * HD:off + (head + 1) * HD], O.bf16_bits_to_f32(kn_bits), pos,
                            invf_t().numpy(), RD, 1e-6, 1.0)
    j = head - NKV
    return p[row, off + NKV * HD + j * HD:off + NKV * HD + (j + 1) * HD]


# ---------------------------------------------------------------- qk_norm_rope
@pytest.mark.parametrize("T,pos0,int8,batch,device_pos", [(1, 0, False, False, False), (5, 17, False, False, False),
                                                         (3, 1000, True, False, False), (4, 1024, True, True, False),
                                                         (4, 1024, True, True, True), (2, 9, False, True, True)])
def test_qk_norm_rope_vs_oracle(pkg, dev, T, pos0, int8, batch, device_pos):
    g = torch.Generator().manual_seed(2000 + T + pos0)
    P = 2 * NQ * HD + 2 * NKV * HD
    proj = rand_bf16(g, (T, P + 256), 0.5)
    qn, kn = rand_bf16(g, (HD,), 0.2), rand_bf16(g, (HD,), 0.2)
    seq = pos0 + T + 3
    rows = T * seq if batch else seq
    kvc = torch.zeros(rows, 2 * NKV * HD, dtype=torch.int8 if int8 else torch.bfloat16, device=dev)
    kvs = torch.zeros(rows, 2 * NKV, device=dev) if int8 else None
    qout = torch.empty(T, NQ * HD, dtype=torch.bfloat16, device=dev)
    pos_arg = torch.tensor([pos0], dtype=torch.int32, device=dev) if device_pos else pos0
    pkg.qk_norm_rope(proj.to(dev), qn.to(dev), kn.to(dev), invf_t().to(dev), qout, kvc, kvs, pos_arg, 1e-6,
                     kv_int8=int8, batch=batch, kv_stride=seq * 2 * NKV * HD if batch else None,
                     kvs_stride=seq * 2 * NKV if batch else None)
    torch.cuda.synchronize()
    ref_kvc = np.zeros((rows, 2 * NKV * HD), dtype=np.int8 if int8 else np.uint16)
    ref_kvs = np.zeros((rows, 2 * NKV), dtype=np.float32) if int8 else None
    rq = O.qk_norm_rope(bits(proj), bits(qn), bits(kn), invf_t().numpy(), NQ, NKV, HD, pos0, ref_kvc, ref_kvs,
                        batch=batch)
    assert_bf16_close(bits(qout), rq, "q")
    got = kvc.cpu().numpy() if int8 else bits(kvc)
    for t in range(T):
        pos = pos0 if batch else pos0 + t
        r = (t * seq if batch else 0) + pos
        for head in range(2 * NKV):
            sl = slice(head * HD, (head + 1) * HD)
            if int8:
                y = oracle_kv(bits(proj), bits(kn), 0, t, pos, head)
                assert_kv_codes(got[r:r + 1, sl], kvs.cpu().numpy()[r:r + 1, head], y[None, :], f"kv row {r} h{head}")
            else:
                assert_bf16_close(got[r:r + 1, sl], ref_kvc[r:r + 1, sl], f"kv row {r} h{head}")
    # no other cache row was touched
    written = {(t * seq if batch else 0) + (pos0 if batch else pos0 + t) for t in range(T)}
    other = [i for i in range(rows) if i not in written]
    assert not np.any(got[other]), "cache rows outside the written positions changed"


@pytest.mark.parametrize("i", ["0", "1", "2"])
def test_qk_norm_rope_vs_reference_golden(pkg, dev, i):
    p = f"qk_rope_{i}_"
    T, pos0, int8, batch, seq = (int(v) for v in GOLD[p + "cfg"])
    rows = T * seq if batch else seq
    kvc = torch.zeros(rows, 2 * NKV * HD, dtype=torch.int8 if int8 else torch.bfloat16, device=dev)
    kvs = torch.zeros(rows, 2 * NKV, device=dev) if int8 else None
    qout = torch.empty(T, NQ * HD, dtype=torch.bfloat16, device=dev)
    pkg.qk_norm_rope(from_bits(GOLD[p + "proj"]).to(dev), from_bits(GOLD[p + "qn"]).to(dev),
                     from_bits(GOLD[p + "kn"]).to(dev), torch.from_numpy(GOLD[p + "invf"]).to(dev), qout, kvc, kvs,
                     pos0, kv_int8=bool(int8), batch=bool(batch), kv_stride=seq * 2 * NKV * HD if batch else None,
                     kvs_stride=seq * 2 * NKV if batch else None)
    torch.cuda.synchronize()
    # the golden q is bf16-truncated (CPU interpreter): within the bar of it
    assert_bf16_close(bits(qout), GOLD[p + "q"], f"golden q {i}")
    if int8:
        d = kvc.cpu().numpy().astype(np.int32) - GOLD[p + "kvc"].astype(np.int32)
        assert np.abs(d).max() <= 1 and (d != 0).mean() < 1e-3
        np.testing.assert_allclose(kvs.cpu().numpy(), GOLD[p + "kvs"], rtol=1e-5)
    else:
        assert_bf16_close(bits(kvc), GOLD[p + "kvc"], f"golden kv {i}")


# ---------------------------------------------------------------- attn_decode
def _cache(g, B, S, int8):
    if int8:
        kvc = torch.randint(-127, 128, (B * S, 2 * NKV * HD), dtype=torch.int8, generator=g)
        kvs = torch.rand(B * S, 2 * NKV, generator=g) * 0.02 + 0.001
        return kvc, kvs
    return rand_bf16(g, (B * S, 2 * NKV * HD)), None


@pytest.mark.parametrize("B,pos,int8,device_pos", [(1, 0, False, False), (1, 40, False, False), (1, 63, True, False),
                                                   (4, 1024, True, False), (4, 1024, True, True),
                                                   (3, 700, False, True), (2, 5000, True, False)])
def test_attn_decode_vs_oracle(pkg, dev, B, pos, int8, device_pos):
    g = torch.Generator().manual_seed(2100 + B + pos)
    S = pos + 7
    q = rand_bf16(g, (B, NQ * HD), 0.1)
    kvc, kvs = _cache(g, B, S, int8)
    out = torch.empty(B, NQ * HD, dtype=torch.bfloat16, device=dev)
    pos_arg = torch.tensor([pos], dtype=torch.int32, device=dev) if device_pos else pos
    pkg.attn_decode(q.to(dev) if B > 1 else q.to(dev)[0], kvc.to(dev), out if B > 1 else out[0], pos_arg,
                    kvs=None if kvs is None else kvs.to(dev), kv_int8=int8, batch=B, nq=NQ, nkv=NKV, hd=HD)
    ref = O.attn_decode(bits(q), kvc.numpy() if int8 else bits(kvc), pos, None if kvs is None else kvs.numpy(),
                        batch=B)
    assert_bf16_close(bits(out), ref, f"attn_decode B={B} pos={pos}")


@pytest.mark.parametrize("i", ["0", "1", "2"])
def test_attn_decode_vs_reference_golden(pkg, dev, i):
    p = f"attn_decode_{i}_"
    B, pos, int8 = (int(v) for v in GOLD[p + "cfg"])
    kvc = torch.from_numpy(GOLD[p + "kvc"]) if int8 else from_bits(GOLD[p + "kvc"])
    kvs = torch.from_numpy(GOLD[p + "kvs"]).to(dev) if int8 else None
    out = torch.empty(B, NQ * HD, dtype=torch.bfloat16, device=dev)
    pkg.attn_decode(from_bits(GOLD[p + "q"]).to(dev), kvc.to(dev), out, pos, kvs=kvs, kv_int8=bool(int8), batch=B,
                    nq=NQ, nkv=NKV, hd=HD)
    assert_bf16_close(bits(out), GOLD[p + "out"], f"golden attn {i}")


def test_attn_decode_graph_replay_at_moving_position(pkg, dev):
    """One captured launch, replayed with the device-side position advanced
    in place: each replay matches the oracle at its position."""
    g = torch.Generator().manual_seed(2150)
    B, S = 2, 300
    q = rand_bf16(g, (B, NQ * HD), 0.1).to(dev)
    kvc, kvs = _cache(g, B, S, True)
    kvc_d, kvs_d = kvc.to(dev), kvs.to(dev)
    out = torch.empty(B, NQ * HD, dtype=torch.bfloat16, device=dev)
    pos = torch.tensor([10], dtype=torch.int32, device=dev)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        pkg.attn_decode(q, kvc_d, out, pos, kvs=kvs_d, kv_int8=True, batch=B, max_pos=S - 1)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        pkg.attn_decode(q, kvc_d, out, pos, kvs=kvs_d, kv_int8=True, batch=B, max_pos=S - 1)
    for p_ in (0, 63, 64, 257, 299):
        pos.fill_(p_)
        graph.replay()
        torch.cuda.synchronize()
        ref = O.attn_decode(bits(q), kvc.numpy(), p_, kvs.numpy(), batch=B)
        assert_bf16_close(bits(out), ref, f"replay pos={p_}")


# ---------------------------------------------------------------- delta_decode
def _state_close(got, ref, what):
    err = np.abs(got - ref)
    bad = err > 1e-6 + 1e-5 * np.abs(ref)
    assert not bad.any(), f"{what}: {int(bad.sum())} state values outside the bar, max err {err.max()}"


@pytest.mark.parametrize("B", [1, 4])
def test_delta_decode_vs_oracle(pkg, dev, B):
    g = torch.Generator().manual_seed(2200 + B)
    qkv = rand_bf16(g, (B, CONV + 512), 0.3)     # a row of a wider buffer (engine.py:226)
    gg = -torch.rand(B, NH, generator=g) * 0.4
    beta = torch.rand(B, NH, generator=g)
    state = torch.randn(B * NH, DK, DV, generator=g) * 0.05
    st = state.to(dev)
    out = torch.empty(B, NH * DV, dtype=torch.bfloat16, device=dev)
    qd = qkv.to(dev)[:, :CONV]
    if B == 1:
        pkg.delta_decode(qd[0], gg.to(dev)[0], beta.to(dev)[0], st, out[0])
    else:
        pkg.delta_decode(qd, gg.to(dev), beta.to(dev), st, out, batch=B)
    ref_state = state.numpy().copy()
    ref = O.delta_decode(bits(qkv[:, :CONV]), gg.numpy(), beta.numpy(), ref_state)
    assert_bf16_close(bits(out), ref, f"delta_decode B={B}")
    _state_close(st.cpu().numpy(), ref_state, f"delta state B={B}")


@pytest.mark.parametrize("i", ["0", "1"])
def test_delta_decode_vs_reference_golden(pkg, dev, i):
    p = f"delta_decode_{i}_"
    qkv = from_bits(GOLD[p + "qkv"]).to(dev)
    B = qkv.shape[0]
    st = torch.from_numpy(GOLD[p + "state"].copy()).to(dev)
    out = torch.empty(B, NH * DV, dtype=torch.bfloat16, device=dev)
    gg, beta = torch.from_numpy(GOLD[p + "g"]).to(dev), torch.from_numpy(GOLD[p + "beta"]).to(dev)
    pkg.delta_decode(qkv, gg, beta, st, out, batch=B)
    assert_bf16_close(bits(out), GOLD[p + "out"], f"golden delta {i}")
    _state_close(st.cpu().numpy()[:2], GOLD[p + "state_out2"], f"golden delta state {i}")


# ---------------------------------------------------------------- conv
@pytest.mark.parametrize("T,batch", [(1, False), (2, False), (23, False), (4, True), (1, True)])
def test_conv_vs_oracle(pkg, dev, T, batch):
    g = torch.Generator().manual_seed(2300 + T)
    xw = rand_bf16(g, (T, CONV + 2048))          # x is a column slice of the projection row
    w = rand_bf16(g, (CONV, 4), 0.1)
    state = rand_bf16(g, (3 * T if batch else 3, CONV))
    xd = xw.to(dev)[:, :CONV]
    sd = state.to(dev)
    y = torch.empty(T, CONV, dtype=torch.bfloat16, device=dev)
    pkg.conv_silu(xd, w.to(dev), sd, y, T, batch=batch)
    pkg.conv_state_update(xd, sd, T, batch=T if batch else 1)
    torch.cuda.synchronize()
    xb = bits(xw[:, :CONV].contiguous())
    assert_bf16_close(bits(y), O.conv_silu(xb, bits(w), bits(state), T, batch=batch), f"conv T={T}")
    np.testing.assert_array_equal(bits(sd), O.conv_state_update(xb, bits(state), T, batch=T if batch else 1))


@pytest.mark.parametrize("i", ["0", "1", "2"])
def test_conv_vs_reference_golden(pkg, dev, i):
    p = f"conv_{i}_"
    T, batch = (int(v) for v in GOLD[p + "cfg"])
    x = from_bits(GOLD[p + "x"]).to(dev)
    st = from_bits(GOLD[p + "state"]).to(dev)
    y = torch.empty_like(x)
    pkg.conv_silu(x, from_bits(GOLD[p + "w"]).to(dev), st, y, T, batch=bool(batch))
    pkg.conv_state_update(x, st, T, batch=T if batch else 1)
    torch.cuda.synchronize()
    assert_bf16_close(bits(y), GOLD[p + "y"], f"golden conv {i}")
    np.testing.assert_array_equal(bits(st), GOLD[p + "state_out"])


@pytest.mark.parametrize("B", [1, 4])
def test_conv_silu_update_equals_the_two_calls(pkg, dev, B):
    g = torch.Generator().manual_seed(2350 + B)
    xw = rand_bf16(g, (B, CONV + 2048)).to(dev)
    x = xw[:, :CONV]
    w = rand_bf16(g, (CONV, 4), 0.1).to(dev)
    state = rand_bf16(g, (3 * B, CONV)).to(dev)
    s1, s2 = state.clone(), state.clone()
    y1 = torch.empty(B, CONV, dtype=torch.bfloat16, device=dev)
    y2 = torch.empty_like(y1)
    pkg.conv_silu(x, w, s1, y1, B, batch=True)
    pkg.conv_state_update(x, s1, B, batch=B)
    pkg.kernels.linear_attn.conv_silu_update(x, w, s2, y2, B)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(s1, s2)
