"""Batched decode step of the hybrid stack (engine.py:342-375 call pattern)
entirely on this package's kernels.

* A small stack (3 linear-attention layers + 1 full-attention layer, the
  reference's head sizes, hidden 256) against the same step composed from the
  CPU oracle's functions: every per-kernel rounding rule holds layer by layer,
  but int8 requantisation between layers lets a +-1 code at one layer move
  later values slightly, so the comparison is the relative L2 error of the
  logits, the delta-rule state and the written KV row (< 1e-2).
* The whole step captured once in a CUDA graph and replayed at two positions
  (device-side position) equals eager steps bit for bit.
"""
import numpy as np
import pytest
import torch

from oracle import qlin_oracle as O
from qlin_testutil import assert_bf16_close, bits

pytestmark = pytest.mark.gpu

TINY = dict(hidden=256, inter=512, layers=4, pattern=("linear", "linear", "linear", "full"), nh=16, dk=128,
            dv=128, conv=4, nq=8, nkv=2, hd=256, rotary=0.25, rope_theta=1e7, vocab=1024, eps=1e-6)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


def f32(t):
    return O.bf16_bits_to_f32(bits(t)) if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()


def oracle_step(st, ids, pos, kv, kvs, dstate, cstate):
    """The step of HybridStack.step composed from the oracle's functions
    (numpy state arrays updated in place).  Returns the logits (fp32)."""
    B, H = st.B, st.H
    emb = st.embed.cpu()[ids].float() * st.embed_s.cpu()[ids].float()[:, None]
    hidden = O.f32_to_bf16_bits(emb.numpy())

    def gemm_res(aq, as_, w, hidden_bits):
        return O.gemm_i8(aq, as_, w[0].cpu().numpy(), w[1].cpu().numpy(), hidden_bits)

    li = fi = 0
    invf = st.invf.cpu().numpy()
    for t, L in zip(st.types, st.layers):
        xq, xs = O.rmsnorm_quant(hidden, bits(L["in_norm"]), st.eps)
        if t == "linear":
            segs = [(L["qkv"][0].cpu().numpy(), L["qkv"][1].cpu().numpy(), None),
                    (L["z"][0].cpu().numpy(), L["z"][1].cpu().numpy(), None)]
            proj = O.proj3(xq, xs, segs)
            beta, gate = O.gate_proj(xq, xs, bits(L["b"]), bits(L["a"]), bits(L["dt"]), bits(L["alog"]))
            cst = cstate[li].reshape(B * 3, st.conv_dim)
            mixed_in = proj[:, :st.conv_dim]
            mixed = O.conv_silu(mixed_in, bits(L["conv"]), cst, B, batch=True)
            cstate[li] = O.conv_state_update(mixed_in, cst, B, batch=B).reshape(cstate[li].shape)
            ds = dstate[li].reshape(B * st.NH, st.DK, st.DV)
            dout = O.delta_decode(mixed, gate, beta, ds)
            dstate[li] = ds.reshape(dstate[li].shape)
            aq, as_ = O.norm_gated_quant(dout, proj[:, st.conv_dim:], bits(L["norm_w"]), st.eps)
            hidden = gemm_res(aq, as_, L["out"], hidden)
            li += 1
        else:
            segs = [(L[k][0].cpu().numpy(), L[k][1].cpu().numpy(), None) for k in ("q", "k", "v")]
            proj = O.proj3(xq, xs, segs)
            kvf = kv[fi].reshape(B * st.seq, -1)
            kvsf = kvs[fi].reshape(B * st.seq, -1)
            q = O.qk_norm_rope(proj, bits(L["qn"]), bits(L["kn"]), invf, st.NQ, st.NKV, st.HD, pos, kvf, kvsf,
                               st.eps, batch=True)
            kv[fi] = kvf.reshape(kv[fi].shape)
            kvs[fi] = kvsf.reshape(kvs[fi].shape)
            aout = O.attn_decode(q, kvf, pos, kvsf, batch=B, nq=st.NQ, nkv=st.NKV, hd=st.HD)
            aq, as_ = O.gate_mul_quant(aout, proj, st.HD)
            hidden = gemm_res(aq, as_, L["o"], hidden)
            fi += 1
        hq, hs = O.rmsnorm_quant(hidden, bits(L["post_norm"]), st.eps)
        gq, gs = O.mlp_gate_up_quant(hq, hs, L["gate"][0].cpu().numpy(), L["gate"][1].cpu().numpy(),
                                     L["up"][0].cpu().numpy(), L["up"][1].cpu().numpy())
        hidden = gemm_res(gq, gs, L["down"], hidden)
    xq, xs = O.rmsnorm_quant(hidden, bits(st.final_norm), st.eps)
    return O.bf16_bits_to_f32(O.gemm_i8(xq, xs, st.lm_head[0].cpu().numpy(), st.lm_head[1].cpu().numpy()))


def test_decode_step_matches_oracle_composition(pkg, dev):
    B, seq, pos = 2, 20, 13
    st = pkg.decode_step.HybridStack(TINY, dev, B, seq, kv_int8=True, seed=3, init_device="cpu")
    kv, kvs = st.kv.cpu().numpy().copy(), st.kvs.cpu().numpy().copy()
    dstate, cstate = st.dstate.cpu().numpy().copy(), bits(st.cstate).copy()
    ids = torch.tensor([5, 900], device=dev)
    logits = f32(st.step(ids, pos))
    ref = oracle_step(st, ids.cpu(), pos, kv, kvs, dstate, cstate)
    assert rel_l2(logits, ref) < 1e-2, rel_l2(logits, ref)
    assert rel_l2(st.dstate.cpu().numpy(), dstate) < 1e-2
    got_kv = st.kv.cpu().numpy()[:, :, pos].astype(np.float32) * np.repeat(st.kvs.cpu().numpy()[:, :, pos], 256, -1)
    ref_kv = kv[:, :, pos].astype(np.float32) * np.repeat(kvs[:, :, pos], 256, -1)
    assert rel_l2(got_kv, ref_kv) < 1e-2
    # the conv window copies this step's projection rows, which are within the
    # bf16 bar of the oracle's (the copy itself is bit-exact: test_gpu_decode.py)
    assert_bf16_close(bits(st.cstate).reshape(-1, st.conv_dim), cstate.reshape(-1, st.conv_dim), "conv window")


def test_decode_step_graph_replay_equals_eager(pkg, dev):
    B, seq = 2, 40
    ids = torch.tensor([7, 11], device=dev)
    eager = pkg.decode_step.HybridStack(TINY, dev, B, seq, kv_int8=True, seed=4, init_device="cpu")
    graphed = pkg.decode_step.HybridStack(TINY, dev, B, seq, kv_int8=True, seed=4, init_device="cpu")
    pos = torch.tensor([20], dtype=torch.int32, device=dev)
    pos_e = torch.tensor([20], dtype=torch.int32, device=dev)   # same launch plans as the graph's
    graph = graphed.capture(ids, pos, warmup=1)   # one eager step at position 20 before capture
    eager.step(ids, pos_e)
    for p in (21, 22, 35):
        pos.fill_(p)
        pos_e.fill_(p)
        graph.replay()
        out_e = eager.step(ids, pos_e)
        torch.cuda.synchronize()
        assert torch.equal(graphed.logits, out_e), f"position {p}"
        assert torch.equal(graphed.dstate, eager.dstate) and torch.equal(graphed.kv, eager.kv)
        assert torch.equal(graphed.cstate, eager.cstate)
    assert pkg._lib.load().qlin_device_fault(0) == 0
