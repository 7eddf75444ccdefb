// Chunked gated delta-rule prefill (kernels/linear_attn.py:86-169).
//
// CTA = (head h, 32-column slab of V); chunks of 32 tokens in order, the
// state slab S [DK = 128, 32] (fp32) carried in shared memory.  Per chunk,
// in the reference's order (fp32 throughout, as its "ieee" dots):
//   qn = q rsqrt(|q|^2 + 1e-6) / sqrt(DK);  kn = k rsqrt(|k|^2 + 1e-6)
//   gc = cumsum(g);  decay[i, j] = exp(gc_i - gc_j) for i >= j, else 0
//   kb = kn * beta;  A = -(kb kn^T) * decay, strictly lower
//   Tm = (I - A)^-1 by the Neumann product: Tm = I + A, P = A, five times
//        P = P P, Tm = Tm + Tm P
//   value = Tm (v * beta);  kcum = Tm (kb * exp(gc))
//   v_new = value - kcum S
//   out = (qn * exp(gc)) S + ((qn kn^T) * decay) v_new
//   S = S exp(min gc) + (kn * exp(min gc - gc))^T v_new
// Rows past T are zero (q, k, v, beta and g), as the reference's masked loads
// make them.  The products are CUDA-core fp32 with this kernel's own
// summation order.
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kDpChunk = 32, kDpDK = 128, kDpVS = 32, kDpThreads = 256;

struct DeltaPrefillArgs {
  const __nv_bfloat16* qkv;  // [T, ldq]: q [NH*DK], k [NH*DK], v [NH*DV]
  long long ldq;
  const float* g;            // [T, NH]
  const float* beta;         // [T, NH]
  float* state;              // [NH, DK, DV]
  __nv_bfloat16* out;        // [T, NH*DV]
  int T, nh, dv;
};

struct DpSmem {
  float S[kDpDK][kDpVS];
  float q[kDpChunk][kDpDK];
  float k[kDpChunk][kDpDK];
  float kb[kDpChunk][kDpDK];   // kb, then kb * exp(gc)
  float kc[kDpChunk][kDpDK];   // kcum
  float v[kDpChunk][kDpVS];    // v, then v * beta
  float A[kDpChunk][kDpChunk];
  float Tm[kDpChunk][kDpChunk];
  float P[kDpChunk][kDpChunk];
  float decay[kDpChunk][kDpChunk];
  float vn[kDpChunk][kDpVS];
  float qk[kDpChunk][kDpChunk];
  float gc[kDpChunk], eg[kDpChunk], beta[kDpChunk];
  float glast;
};

// C[32 x 32] = A[32 x K] B[K x 32], thread t owns row t/8, columns 4(t%8)..+3.
template <int K, int LDA, int LDB>
__device__ __forceinline__ void dp_mm32(const float* A, const float* B, float (&c)[4]) {
  const int i = threadIdx.x >> 3, j0 = (threadIdx.x & 7) * 4;
  c[0] = c[1] = c[2] = c[3] = 0.0f;
#pragma unroll 8
  for (int kk = 0; kk < K; ++kk) {
    const float a = A[i * LDA + kk];
    const float4 b = *reinterpret_cast<const float4*>(B + kk * LDB + j0);
    c[0] = fmaf(a, b.x, c[0]);
    c[1] = fmaf(a, b.y, c[1]);
    c[2] = fmaf(a, b.z, c[2]);
    c[3] = fmaf(a, b.w, c[3]);
  }
}

__global__ void __launch_bounds__(kDpThreads) delta_prefill_kernel(const __grid_constant__ DeltaPrefillArgs a) {
  extern __shared__ __align__(16) uint8_t dp_raw[];
  DpSmem& s = *reinterpret_cast<DpSmem*>(dp_raw);
  pdl_launch_dependents();
  const int h = blockIdx.x, slab = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int c0 = slab * kDpVS;
  float* Sg = a.state + static_cast<long long>(h) * kDpDK * a.dv;
  pdl_wait();
  for (int i = t; i < kDpDK * kDpVS; i += kDpThreads) s.S[i / kDpVS][i % kDpVS] = Sg[(i / kDpVS) * a.dv + c0 + i % kDpVS];
  const float inv_sqrt_dk = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(kDpDK)));
  const int i8 = t >> 3, j4 = (t & 7) * 4;  // the [32 x 32] product tiling
  for (int ck = 0; ck < a.T; ck += kDpChunk) {
    __syncthreads();
    // load the chunk (rows past T are zero)
    for (int i = t; i < kDpChunk * kDpDK / 8; i += kDpThreads) {
      const int r = i / (kDpDK / 8), c8 = (i % (kDpDK / 8)) * 8;
      float fq[8], fk[8];
      if (ck + r < a.T) {
        const __nv_bfloat16* row = a.qkv + static_cast<long long>(ck + r) * a.ldq;
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + h * kDpDK + c8), fq);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + a.nh * kDpDK + h * kDpDK + c8), fk);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) fq[e] = fk[e] = 0.0f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s.q[r][c8 + e] = fq[e];
        s.k[r][c8 + e] = fk[e];
      }
    }
    for (int i = t; i < kDpChunk * kDpVS; i += kDpThreads) {
      const int r = i / kDpVS, c = i % kDpVS;
      s.v[r][c] = ck + r < a.T
                      ? __bfloat162float(a.qkv[static_cast<long long>(ck + r) * a.ldq + 2 * a.nh * kDpDK + h * a.dv + c0 + c])
                      : 0.0f;
    }
    if (t < kDpChunk) {
      const bool live = ck + t < a.T;
      s.beta[t] = live ? a.beta[static_cast<long long>(ck + t) * a.nh + h] : 0.0f;
      s.gc[t] = live ? a.g[static_cast<long long>(ck + t) * a.nh + h] : 0.0f;
    }
    __syncthreads();
    // l2 norms: warp w normalises rows 4w .. 4w + 3 of q and k
    for (int r = warp * 4; r < warp * 4 + 4; ++r) {
      float sq = 0.0f, sk = 0.0f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float qv = s.q[r][lane * 4 + e], kv = s.k[r][lane * 4 + e];
        sq = __fadd_rn(sq, __fmul_rn(qv, qv));
        sk = __fadd_rn(sk, __fmul_rn(kv, kv));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
        sk = __fadd_rn(sk, __shfl_xor_sync(0xffffffffu, sk, o));
      }
      const float rq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq, 1e-6f)));
      const float rk = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sk, 1e-6f)));
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s.q[r][lane * 4 + e] = __fmul_rn(__fmul_rn(s.q[r][lane * 4 + e], rq), inv_sqrt_dk);
        s.k[r][lane * 4 + e] = __fmul_rn(s.k[r][lane * 4 + e], rk);
      }
    }
    if (t == 0) {  // cumulative sum of g, in order
      float acc = 0.0f, mn = INFINITY;
      for (int r = 0; r < kDpChunk; ++r) {
        acc = __fadd_rn(acc, s.gc[r]);
        s.gc[r] = acc;
        mn = fminf(mn, acc);
      }
      s.glast = mn;
    }
    __syncthreads();
    if (t < kDpChunk) s.eg[t] = expf(s.gc[t]);
    for (int i = t; i < kDpChunk * kDpChunk; i += kDpThreads) {
      const int r = i / kDpChunk, c = i % kDpChunk;
      s.decay[r][c] = r >= c ? expf(__fsub_rn(s.gc[r], s.gc[c])) : 0.0f;
    }
    for (int i = t; i < kDpChunk * kDpDK; i += kDpThreads) {
      const int r = i / kDpDK, c = i % kDpDK;
      s.kb[r][c] = __fmul_rn(s.k[r][c], s.beta[r]);
    }
    for (int i = t; i < kDpChunk * kDpVS; i += kDpThreads) s.v[i / kDpVS][i % kDpVS] =
        __fmul_rn(s.v[i / kDpVS][i % kDpVS], s.beta[i / kDpVS]);
    __syncthreads();
    // A = -(kb kn^T) * decay (strictly lower); qk = (qn kn^T) * decay
    {
      float ca[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
      for (int d = 0; d < kDpDK; ++d) {
        const float kbv = s.kb[i8][d], qv = s.q[i8][d];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float kn = s.k[j4 + e][d];
          ca[e] = fmaf(kbv, kn, ca[e]);
          cq[e] = fmaf(qv, kn, cq[e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = j4 + e;
        const float av = i8 > j ? __fmul_rn(-ca[e], s.decay[i8][j]) : 0.0f;
        s.A[i8][j] = av;
        s.P[i8][j] = av;
        s.Tm[i8][j] = av + (i8 == j ? 1.0f : 0.0f);
        s.qk[i8][j] = __fmul_rn(cq[e], s.decay[i8][j]);
      }
    }
    __syncthreads();
    // Neumann product: P = P P; Tm = Tm + Tm P (five times)
    for (int it = 0; it < 5; ++it) {
      float c[4];
      dp_mm32<kDpChunk, kDpChunk, kDpChunk>(&s.P[0][0], &s.P[0][0], c);
      __syncthreads();
#pragma unroll
      for (int e = 0; e < 4; ++e) s.P[i8][j4 + e] = c[e];
      __syncthreads();
      dp_mm32<kDpChunk, kDpChunk, kDpChunk>(&s.Tm[0][0], &s.P[0][0], c);
      __syncthreads();
#pragma unroll
      for (int e = 0; e < 4; ++e) s.Tm[i8][j4 + e] = __fadd_rn(s.Tm[i8][j4 + e], c[e]);
      __syncthreads();
    }
    // kb * exp(gc) (in place), then value = Tm vb and kcum = Tm (kb e^gc)
    for (int i = t; i < kDpChunk * kDpDK; i += kDpThreads) {
      const int r = i / kDpDK, c = i % kDpDK;
      s.kb[r][c] = __fmul_rn(s.kb[r][c], s.eg[r]);
    }
    __syncthreads();
    float value[4];
    dp_mm32<kDpChunk, kDpChunk, kDpVS>(&s.Tm[0][0], &s.v[0][0], value);
    {
      // kcum [32 x 128]: thread t owns row t/8, columns 16(t%8) .. +15
      const int cc = (t & 7) * 16;
      float kc[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) kc[e] = 0.0f;
#pragma unroll 4
      for (int kk = 0; kk < kDpChunk; ++kk) {
        const float tv = s.Tm[i8][kk];
#pragma unroll
        for (int e = 0; e < 16; ++e) kc[e] = fmaf(tv, s.kb[kk][cc + e], kc[e]);
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) s.kc[i8][cc + e] = kc[e];
    }
    __syncthreads();
    // v_new = value - kcum S
    {
      float c[4];
      dp_mm32<kDpDK, kDpDK, kDpVS>(&s.kc[0][0], &s.S[0][0], c);
#pragma unroll
      for (int e = 0; e < 4; ++e) s.vn[i8][j4 + e] = __fsub_rn(value[e], c[e]);
    }
    // qn * exp(gc), in place (q is not needed otherwise any more)
    for (int i = t; i < kDpChunk * kDpDK; i += kDpThreads) {
      const int r = i / kDpDK, c = i % kDpDK;
      s.q[r][c] = __fmul_rn(s.q[r][c], s.eg[r]);
    }
    __syncthreads();
    // out = (qn e^gc) S + qk v_new
    {
      float c1[4], c2[4];
      dp_mm32<kDpDK, kDpDK, kDpVS>(&s.q[0][0], &s.S[0][0], c1);
      dp_mm32<kDpChunk, kDpChunk, kDpVS>(&s.qk[0][0], &s.vn[0][0], c2);
      if (ck + i8 < a.T) {
        __nv_bfloat16* orow = a.out + static_cast<long long>(ck + i8) * a.nh * a.dv + h * a.dv + c0 + j4;
#pragma unroll
        for (int e = 0; e < 4; ++e) orow[e] = __float2bfloat16_rn(__fadd_rn(c1[e], c2[e]));
      }
    }
    __syncthreads();  // S is read above and rewritten below
    // S = S exp(glast) + (kn exp(glast - gc))^T v_new; thread t owns rows
    // 4(t/8) .. +3 (after t/8 the 32 groups cover 128 rows), columns 4(t%8) .. +3
    {
      const float eg_last = expf(s.glast);
      const int r0 = (t >> 3) * 4;
      float w[kDpChunk];
#pragma unroll
      for (int kk = 0; kk < kDpChunk; ++kk) w[kk] = expf(__fsub_rn(s.glast, s.gc[kk]));
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const int r = r0 + rr;
        float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
        for (int kk = 0; kk < kDpChunk; ++kk) {
          const float kv = __fmul_rn(s.k[kk][r], w[kk]);
          const float4 vn = *reinterpret_cast<const float4*>(&s.vn[kk][j4]);
          c[0] = fmaf(kv, vn.x, c[0]);
          c[1] = fmaf(kv, vn.y, c[1]);
          c[2] = fmaf(kv, vn.z, c[2]);
          c[3] = fmaf(kv, vn.w, c[3]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) s.S[r][j4 + e] = __fadd_rn(__fmul_rn(s.S[r][j4 + e], eg_last), c[e]);
      }
    }
  }
  __syncthreads();
  for (int i = t; i < kDpDK * kDpVS; i += kDpThreads) Sg[(i / kDpVS) * a.dv + c0 + i % kDpVS] = s.S[i / kDpVS][i % kDpVS];
}

}  // namespace qlin
