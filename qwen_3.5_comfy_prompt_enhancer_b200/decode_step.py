"""Batched decode step of a Qwen3.5 hybrid stack on this package's kernels.

``HybridStack`` holds a random-initialised stack of the reference engine's
shapes and layouts (W8 per-channel linears from ``N(0, 0.02)`` quantised as
quant_formats.py:270-275 does, int8 embedding with per-row scales, int8 or
bf16 KV cache, fp32 delta-rule state, bf16 conv windows) and runs the
engine's batched decode step, ``Engine.forward_batch`` (engine.py:342-375):
B candidates at one shared position, every layer through the same kernel
calls as engine.py:291-340 -- rmsnorm_quant, proj3, gate_proj, conv_silu and
conv_state_update (in one launch), delta_decode, norm_gated_quant, qk_norm_rope, attn_decode,
gate_mul_quant, mlp_gate_up_quant, gemm_i8 with the residual in place -- and
the int8 lm_head.  Every kernel is this package's own (the embedding gather is
two torch ops, as in the engine).

The position can live in a one-element int32 CUDA tensor, read by the
kernels at run time, so ``capture`` records the whole step (about 270
launches) in one CUDA graph that replays at any position.

This is the workload of the decode-step benchmark, not a port of the
reference engine: no prefill, sampling, tokenizer or weight loading.
"""
import torch

from .kernels import attention, gemm, linear_attn, norm
from .kernels.common import GROUP

QWEN35_2B = dict(hidden=2048, inter=6144, layers=24, pattern=("linear", "linear", "linear", "full"), nh=16,
                 dk=128, dv=128, conv=4, nq=8, nkv=2, hd=256, rotary=0.25, rope_theta=1e7, vocab=151936, eps=1e-6)


def requant_w8_row(w):
    """float [K, N] -> (int8 [K, N], fp32 scale [N]) per-column symmetric
    (quant_formats.py:270-275)."""
    amax = w.abs().amax(dim=0).clamp_min(1e-8)
    sc = (amax / 127.0).float()
    q = torch.clamp(torch.round(w / sc[None, :]), -127, 127).to(torch.int8)
    return q, sc


class HybridStack:
    """Random-initialised hybrid stack (``cfg`` shapes) on ``device`` with
    decode state for ``batch`` candidates and ``seq`` cache positions."""

    def __init__(self, cfg, device, batch, seq, kv_int8=True, seed=0, init_device=None):
        self.cfg = c = dict(cfg)
        self.device = d = torch.device(device)
        gd = torch.device(init_device) if init_device is not None else d
        g = torch.Generator(device=gd).manual_seed(seed)
        self.B, self.seq, self.kv_int8 = batch, seq, kv_int8
        H, I, V = c["hidden"], c["inter"], c["vocab"]
        NH, DK, DV, NQ, NKV, HD = c["nh"], c["dk"], c["dv"], c["nq"], c["nkv"], c["hd"]
        self.H, self.I, self.V, self.NH, self.DK, self.DV = H, I, V, NH, DK, DV
        self.NQ, self.NKV, self.HD = NQ, NKV, HD
        self.conv_dim = 2 * NH * DK + NH * DV
        self.types = [c["pattern"][i % len(c["pattern"])] for i in range(c["layers"])]
        self.eps = c["eps"]
        rd = int(HD * c["rotary"])
        self.invf = (1.0 / (c["rope_theta"] ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))).to(d)

        def lin(k, n):
            q, s = requant_w8_row(torch.randn(k, n, device=gd, generator=g) * 0.02)
            return q.to(d), s.to(d)

        def vec(n, scale=0.1, shift=0.0):
            return (torch.randn(n, device=gd, generator=g) * scale + shift).to(torch.bfloat16).to(d)

        self.layers = []
        for t in self.types:
            L = {"in_norm": vec(H), "post_norm": vec(H),
                 "gate": lin(H, I), "up": lin(H, I), "down": lin(I, H)}
            if t == "linear":
                L.update(qkv=lin(H, self.conv_dim), z=lin(H, NH * DV), out=lin(NH * DV, H),
                         b=vec(NH * H, 0.02).view(NH, H), a=vec(NH * H, 0.02).view(NH, H),
                         dt=vec(NH, 1.0), alog=vec(NH, 0.5), conv=vec(self.conv_dim * c["conv"], 0.2).view(
                             self.conv_dim, c["conv"]), norm_w=vec(DV, 0.1, 1.0))
            else:
                L.update(q=lin(H, NQ * HD * 2), k=lin(H, NKV * HD), v=lin(H, NKV * HD), o=lin(NQ * HD, H),
                         qn=vec(HD), kn=vec(HD))
            self.layers.append(L)
        self.final_norm = vec(H)
        eq, es = requant_w8_row(torch.randn(H, V, device=gd, generator=g) * 0.02)
        self.lm_head = (eq.to(d), es.to(d))
        # int8 embedding, one bf16 scale per vocabulary row (weights.py:421-432)
        emb = torch.randn(V, H, device=gd, generator=g) * 0.02
        amax = emb.abs().amax(dim=1).clamp_min(1e-8)
        self.embed_s = (amax / 127.0).to(torch.bfloat16).to(d)
        self.embed = torch.clamp(torch.round(emb / (amax / 127.0)[:, None]), -127, 127).to(torch.int8).to(d)
        del emb
        # decode state of `batch` candidates (engine.py:413-425 layouts)
        n_lin = self.types.count("linear")
        n_full = len(self.types) - n_lin
        kv_dim = 2 * NKV * HD
        if kv_int8:
            self.kv = torch.randint(-127, 128, (n_full, batch, seq, kv_dim), dtype=torch.int8, device=gd,
                                    generator=g).to(d)
            self.kvs = (torch.rand(n_full, batch, seq, 2 * NKV, device=gd, generator=g) * 0.02 + 1e-3).to(d)
        else:
            self.kv = (torch.randn(n_full, batch, seq, kv_dim, device=gd, generator=g) * 0.5).to(torch.bfloat16).to(d)
            self.kvs = None
        self.dstate = (torch.randn(n_lin, batch, NH, DK, DV, device=gd, generator=g) * 0.05).to(d)
        self.cstate = (torch.randn(n_lin, batch, c["conv"] - 1, self.conv_dim, device=gd, generator=g)).to(
            torch.bfloat16).to(d)
        # workspace rows (engine.py:28-66)
        B = batch
        e = dict(device=d)
        self.hidden = torch.empty(B, H, dtype=torch.bfloat16, **e)
        self.eq = torch.empty(B, H, dtype=torch.int8, **e)
        self.xq = torch.empty(B, H, dtype=torch.int8, **e)
        self.xs = torch.empty(B, H // GROUP, dtype=torch.float32, **e)
        self.proj = torch.empty(B, max(self.conv_dim + NH * DV, NQ * HD * 2 + 2 * NKV * HD), dtype=torch.bfloat16,
                                **e)
        self.mixed = torch.empty(B, self.conv_dim, dtype=torch.bfloat16, **e)
        self.dout = torch.empty(B, NH * DV, dtype=torch.bfloat16, **e)
        self.aq_o = torch.empty(B, NQ * HD, dtype=torch.int8, **e)
        self.as_o = torch.empty(B, NQ * HD // GROUP, dtype=torch.float32, **e)
        self.lq = torch.empty(B, NH * DV, dtype=torch.int8, **e)
        self.ls = torch.empty(B, NH * DV // GROUP, dtype=torch.float32, **e)
        self.q = torch.empty(B, NQ * HD, dtype=torch.bfloat16, **e)
        self.aout = torch.empty(B, NQ * HD, dtype=torch.bfloat16, **e)
        self.hq = torch.empty(B, I, dtype=torch.int8, **e)
        self.hs = torch.empty(B, I // GROUP, dtype=torch.float32, **e)
        self.beta = torch.empty(B, NH, dtype=torch.float32, **e)
        self.gate = torch.empty(B, NH, dtype=torch.float32, **e)
        self.logits = torch.empty(B, V, dtype=torch.bfloat16, **e)
        # kernel launches of one step (the embedding's two torch ops aside)
        self.launches = sum(7 if t == "linear" else 6 for t in self.types) + 3 * len(self.types) + 2

    # ------------------------------------------------------------------ layers
    def _linear(self, L, li, pos):
        B = self.B
        norm.rmsnorm_quant(self.hidden, L["in_norm"], self.xq, self.xs, self.eps)
        gemm.proj3(self.xq, self.xs, L["qkv"][0], L["qkv"][1], L["z"][0], L["z"][1], None, None, self.proj)
        norm.gate_proj(self.xq, self.xs, L["b"], L["a"], self.beta, self.gate, L["dt"], L["alog"])
        mixed_in = self.proj[:, :self.conv_dim]
        cst = self.cstate[li].view(B * (self.cfg["conv"] - 1), self.conv_dim)
        # conv_silu + conv_state_update (engine.py:302-303) in one launch
        linear_attn.conv_silu_update(mixed_in, L["conv"], cst, self.mixed, B)
        dst = self.dstate[li].view(B * self.NH, self.DK, self.DV)
        linear_attn.delta_decode(self.mixed, self.gate, self.beta, dst, self.dout, batch=B)
        norm.norm_gated_quant(self.dout, self.proj[:, self.conv_dim:], L["norm_w"], self.lq, self.ls, self.eps)
        gemm.gemm_i8(self.lq, self.ls, L["out"][0], L["out"][1], self.hidden, residual=self.hidden)

    def _attn(self, L, fi, pos):
        B, seq = self.B, self.seq
        norm.rmsnorm_quant(self.hidden, L["in_norm"], self.xq, self.xs, self.eps)
        gemm.proj3(self.xq, self.xs, L["q"][0], L["q"][1], L["k"][0], L["k"][1], L["v"][0], L["v"][1], self.proj)
        kv_flat = self.kv[fi].view(B * seq, 2 * self.NKV * self.HD)
        kvs_flat = self.kvs[fi].view(B * seq, 2 * self.NKV) if self.kvs is not None else None
        attention.qk_norm_rope(self.proj, L["qn"], L["kn"], self.invf, self.q, kv_flat, kvs_flat, pos, self.eps,
                               kv_int8=self.kv_int8, batch=True, kv_stride=seq * 2 * self.NKV * self.HD,
                               kvs_stride=seq * 2 * self.NKV)
        attention.attn_decode(self.q, kv_flat, self.aout, pos, kvs=kvs_flat, kv_int8=self.kv_int8, batch=B,
                              nq=self.NQ, nkv=self.NKV, hd=self.HD, max_pos=seq - 1)
        norm.gate_mul_quant(self.aout, self.proj, self.aq_o, self.as_o, hd=self.HD)
        gemm.gemm_i8(self.aq_o, self.as_o, L["o"][0], L["o"][1], self.hidden, residual=self.hidden)

    def _mlp(self, L):
        norm.rmsnorm_quant(self.hidden, L["post_norm"], self.xq, self.xs, self.eps)
        gemm.mlp_gate_up_quant(self.xq, self.xs, L["gate"][0], L["gate"][1], L["up"][0], L["up"][1], self.hq,
                               self.hs)
        gemm.gemm_i8(self.hq, self.hs, L["down"][0], L["down"][1], self.hidden, residual=self.hidden)

    def step(self, ids, pos):
        """One batched decode step (engine.py:342-375): ``ids`` int64 CUDA
        tensor [B] of token ids, ``pos`` the shared position (int, or a
        one-element int32 CUDA tensor read at run time).  Returns the logits
        buffer [B, V] (bf16), overwritten by the next step."""
        torch.index_select(self.embed, 0, ids, out=self.eq)
        sc = self.embed_s.index_select(0, ids).unsqueeze(1)
        torch.mul(self.eq, sc, out=self.hidden)
        li = fi = 0
        for t, L in zip(self.types, self.layers):
            if t == "linear":
                self._linear(L, li, pos)
                li += 1
            else:
                self._attn(L, fi, pos)
                fi += 1
            self._mlp(L)
        norm.rmsnorm_quant(self.hidden, self.final_norm, self.xq, self.xs, self.eps)
        gemm.gemm_i8(self.xq, self.xs, self.lm_head[0], self.lm_head[1], self.logits)
        return self.logits

    def capture(self, ids, pos, warmup=2):
        """CUDA graph of ``step(ids, pos)``; ``pos`` must be a device tensor
        for the replay to follow later positions written into it."""
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(ids, pos)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.step(ids, pos)
        return graph

    # ------------------------------------------------------------------ accounting
    def weight_bytes(self):
        """int8 weights + fp32 scales of every projection and the lm_head (the
        streamed bytes of one step; norms, gates and the conv taps aside)."""
        n = 0
        for L in self.layers:
            for k, v in L.items():
                if isinstance(v, tuple):
                    n += v[0].numel() + v[1].numel() * 4
        return n + self.lm_head[0].numel() + self.lm_head[1].numel() * 4

    def step_bytes(self, pos):
        """Algorithmic HBM bytes of one step at `pos`: weights, the delta-rule
        state read + written, the KV cache read (positions 0..pos) and written."""
        n_lin = self.types.count("linear")
        n_full = len(self.types) - n_lin
        state = 2 * n_lin * self.B * self.NH * self.DK * self.DV * 4
        kv_row = 2 * self.NKV * self.HD * (1 if self.kv_int8 else 2) + (2 * self.NKV * 4 if self.kv_int8 else 0)
        kv = n_full * self.B * (pos + 1) * kv_row
        return self.weight_bytes() + state + kv
