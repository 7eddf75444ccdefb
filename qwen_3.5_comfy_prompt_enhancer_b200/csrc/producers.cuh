// Activation producers of the quantised-linear path: the kernels that turn
// the residual stream, the attention output and the linear-attention output
// into the int8 codes + per-64 fp32 scales (a_q, a_s) every GEMM consumes
// (kernels/norm.py of the reference), and the linear-attention gate
// projection that reads those codes (norm.py:211-240).
//
// All are HBM/latency-bound elementwise + row-reduction work: 16-byte
// vector loads of 8 bf16 per lane, fp32 arithmetic in the reference's order,
// one warp-shuffle amax per 64-element group over the 8 lanes (or fewer) that
// hold it, IEEE division for the scale and the codes:
//   s = max(amax / 127, 1e-8),  q = round_half_away(y / s)   (norm.py:15-25).
// Sums of squares are fp32 but their order (per-lane, then warp tree, then
// across warps) is this kernel's own; the reference's order is its
// compiler's, so integer codes can only differ where a value sits on a
// rounding boundary that the last bit of the sum decides.
//
// PDL: each kernel lets the next launch be placed at once and reads its
// activation inputs only after the grid dependency resolves; weights (norm
// and projection weights, read-only model parameters) may be read before.
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kProdThreads = 256;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& raw, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Sigmoid as Triton writes it (triton.language.standard.sigmoid):
// 1 / (1 + exp(-x)), IEEE division, library expf.
__device__ __forceinline__ float sigmoid_ref(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// softplus (kernels/common.py:37-39): x > 20 ? x : log(1 + exp(min(x, 20))).
__device__ __forceinline__ float softplus_ref(float x) {
  return x > 20.0f ? x : logf(__fadd_rn(1.0f, expf(fminf(x, 20.0f))));
}

// 1 / sqrt(v) with a correctly rounded square root and division (the value
// the reference computes as tl.rsqrt(v) under its CPU interpreter).
__device__ __forceinline__ float rsqrt_ieee(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

// Quantise 8 values of a 64-element group held by LG lanes (LG = 8: lanes
// 8j..8j+7 of the warp hold group j, 8 values each).  Every lane of the warp
// takes part in the shuffles; only `valid` lanes store.  Codes go to q8 (8
// bytes, 8-byte aligned), the group's scale to *sc by the group's first lane.
template <int LG>
__device__ __forceinline__ void quant_group_store(const float (&v)[8], bool valid, int8_t* q8, float* sc_dst,
                                                  bool first) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = LG / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (!valid) return;
  const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
  uint32_t packed[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t b = static_cast<uint8_t>(round_i8(__fdiv_rn(v[i], sc)));
    packed[i >> 2] |= b << (8 * (i & 3));
  }
  *reinterpret_cast<uint2*>(q8) = make_uint2(packed[0], packed[1]);
  if (first) *sc_dst = sc;
}

// Sum over the CTA (kProdThreads threads); every thread gets the total.
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kProdThreads / 32; ++i) t = __fadd_rn(t, red[i]);
  return t;
}

// ---------------------------------------------------------------- rmsnorm_quant
// kernels/norm.py:28-57.  One CTA per row; thread t owns the 8-element chunks
// t, t + 256, ... (NV of them) in registers.
//   var = sum(x^2) / K;  y = x * rsqrt(var + eps) * w   (w + 1 with one_plus)
template <int NV>
__global__ void __launch_bounds__(kProdThreads) rmsnorm_quant_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w, int K, float eps,
    int one_plus, int8_t* __restrict__ q, float* __restrict__ s) {
  __shared__ float red[kProdThreads / 32];
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int nch = K / 8;
  float wv[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = threadIdx.x + i * kProdThreads;
    if (c < nch) {
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(w + 8 * c), wv[i]);
      if (one_plus) {
#pragma unroll
        for (int j = 0; j < 8; ++j) wv[i][j] = __fadd_rn(wv[i][j], 1.0f);
      }
    }
  }
  pdl_wait();
  float xv[NV][8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = threadIdx.x + i * kProdThreads;
    if (c < nch) {
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(x + row * ldx + 8 * c), xv[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(xv[i][j], xv[i][j]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[i][j] = 0.0f;
    }
  }
  const float var = __fdiv_rn(cta_sum(ss, red), static_cast<float>(K));
  const float r = rsqrt_ieee(__fadd_rn(var, eps));
  const int G = K / kGroup;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = threadIdx.x + i * kProdThreads;
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = c < nch ? __fmul_rn(__fmul_rn(xv[i][j], r), wv[i][j]) : 0.0f;
    quant_group_store<8>(y, c < nch, q + static_cast<long long>(row) * K + 8 * c,
                         s + static_cast<long long>(row) * G + c / 8, (c & 7) == 0);
  }
}

// ---------------------------------------------------------------- norm_gated(_quant)
// kernels/norm.py:95-165.  One warp per (token, head) of HD dims; lane l owns
// E = HD / 32 consecutive dims.
//   var = sum(x^2) / HD;  y = x * rsqrt(var + eps) * w * silu(z)
// QUANT: y rounded through bf16, then per-64 quantisation within the head;
// otherwise y stored as bf16.
template <int HD, bool QUANT>
__global__ void __launch_bounds__(kProdThreads) norm_gated_kernel(
    const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ z, long long ldz,
    const __nv_bfloat16* __restrict__ w, int T, int NV, float eps, int8_t* __restrict__ q, float* __restrict__ s,
    __nv_bfloat16* __restrict__ out) {
  constexpr int E = HD / 32;            // dims per lane: 2, 4 or 8
  constexpr int LG = kGroup / E;        // lanes per 64-dim group
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long item = static_cast<long long>(blockIdx.x) * (kProdThreads / 32) + warp;
  const bool live = item < static_cast<long long>(T) * NV;
  const int t = live ? static_cast<int>(item / NV) : 0, h = live ? static_cast<int>(item % NV) : 0;
  float wv[E];
  {
    const __nv_bfloat16* wp = w + lane * E;
#pragma unroll
    for (int j = 0; j < E; ++j) wv[j] = __bfloat162float(wp[j]);
  }
  pdl_wait();
  float xv[E], zv[E];
  float ss = 0.0f;
  if (live) {
    const __nv_bfloat16* vp = v + (static_cast<long long>(t) * NV + h) * HD + lane * E;
    const __nv_bfloat16* zp = z + static_cast<long long>(t) * ldz + h * HD + lane * E;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      xv[j] = __bfloat162float(vp[j]);
      zv[j] = __bfloat162float(zp[j]);
      ss = __fadd_rn(ss, __fmul_rn(xv[j], xv[j]));
    }
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) xv[j] = zv[j] = 0.0f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float r = rsqrt_ieee(__fadd_rn(__fdiv_rn(ss, static_cast<float>(HD)), eps));
  float y[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = 0.0f;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const float sz = __fmul_rn(zv[j], sigmoid_ref(zv[j]));  // silu(z) (kernels/common.py:32-34)
    y[j] = __fmul_rn(__fmul_rn(__fmul_rn(xv[j], r), wv[j]), sz);
  }
  const long long base = (static_cast<long long>(t) * NV + h) * HD + lane * E;
  if constexpr (QUANT) {
#pragma unroll
    for (int j = 0; j < E; ++j) y[j] = bf16_round_f32(y[j]);
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) amax = fmaxf(amax, fabsf(y[j]));
#pragma unroll
    for (int o = LG / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (!live) return;
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    int8_t* qp = q + base;
#pragma unroll
    for (int j = 0; j < E; ++j) qp[j] = round_i8(__fdiv_rn(y[j], sc));
    if ((lane % LG) == 0) s[base / kGroup] = sc;
  } else {
    if (!live) return;
#pragma unroll
    for (int j = 0; j < E; ++j) out[base + j] = __float2bfloat16_rn(y[j]);
  }
}

// ---------------------------------------------------------------- gate_mul_quant / silu_mul_quant
// kernels/norm.py:168-208.  Grid (column blocks of 2048, rows); thread t owns
// one 8-element chunk.
//   GATE_MUL: y = a * sigmoid(g), g the second half of each 2*HD head block
//             of the q projection row: column (n / HD) * 2 HD + HD + n % HD
//   SILU_MUL: y = silu(g) * u
template <bool GATE_MUL>
__global__ void __launch_bounds__(kProdThreads) mul_quant_kernel(
    const __nv_bfloat16* __restrict__ a, long long lda, const __nv_bfloat16* __restrict__ g, long long ldg, int N,
    int HD, int8_t* __restrict__ q, float* __restrict__ s) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.y;
  const int c = blockIdx.x * kProdThreads + threadIdx.x;  // 8-element chunk
  const bool valid = 8 * c < N;
  float y[8];
  if (valid) {
    const int n = 8 * c;
    float av[8], gv[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(a + row * lda + n), av);
    const long long gcol = GATE_MUL ? static_cast<long long>(n / HD) * 2 * HD + HD + n % HD : n;
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(g + row * ldg + gcol), gv);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      y[j] = GATE_MUL ? __fmul_rn(av[j], sigmoid_ref(gv[j])) : __fmul_rn(__fmul_rn(gv[j], sigmoid_ref(gv[j])), av[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = 0.0f;
  }
  quant_group_store<8>(y, valid, q + static_cast<long long>(row) * N + 8 * c,
                       s + static_cast<long long>(row) * (N / kGroup) + c / 8, (c & 7) == 0);
}

// ---------------------------------------------------------------- gate_proj
// kernels/norm.py:211-240: from the int8 activations of one row,
//   x = a_q * a_s;  b = wb @ x;  av = wa @ x  (NB outputs each)
//   beta = sigmoid(b);  g = -exp(A_log) * softplus(av + dt_bias)
// One CTA per (output n, row): thread t owns 8-element chunks of K of both
// weight rows, then the two dot products reduce over the CTA.  (One CTA per
// row streamed both whole [NB, K] matrices through 4 SMs at decode batch 4.)
__global__ void __launch_bounds__(kProdThreads) gate_proj_kernel(
    const int8_t* __restrict__ a_q, const float* __restrict__ a_s, int K, const __nv_bfloat16* __restrict__ wb,
    const __nv_bfloat16* __restrict__ wa, int NB, const __nv_bfloat16* __restrict__ dt_bias,
    const __nv_bfloat16* __restrict__ a_log, float* __restrict__ beta, float* __restrict__ gate) {
  __shared__ float red[2][kProdThreads / 32];
  pdl_launch_dependents();
  const int n = blockIdx.x, row = blockIdx.y;
  const int G = K / kGroup;
  const __nv_bfloat16* wbn = wb + static_cast<long long>(n) * K;
  const __nv_bfloat16* wan = wa + static_cast<long long>(n) * K;
  pdl_wait();
  float accb = 0.0f, acca = 0.0f;
  for (int c = threadIdx.x; 8 * c < K; c += kProdThreads) {
    const uint2 raw = *reinterpret_cast<const uint2*>(a_q + static_cast<long long>(row) * K + 8 * c);
    const float sc = a_s[static_cast<long long>(row) * G + c / 8];
    float fb[8], fa[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(wbn + 8 * c), fb);
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(wan + 8 * c), fa);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t word = j < 4 ? raw.x : raw.y;
      const float x = __fmul_rn(static_cast<float>(static_cast<int8_t>((word >> (8 * (j & 3))) & 0xFF)), sc);
      accb = __fadd_rn(accb, __fmul_rn(fb[j], x));
      acca = __fadd_rn(acca, __fmul_rn(fa[j], x));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    accb = __fadd_rn(accb, __shfl_xor_sync(0xffffffffu, accb, o));
    acca = __fadd_rn(acca, __shfl_xor_sync(0xffffffffu, acca, o));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][warp] = accb;
    red[1][warp] = acca;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.0f, av = 0.0f;
#pragma unroll
    for (int i = 0; i < kProdThreads / 32; ++i) {
      b = __fadd_rn(b, red[0][i]);
      av = __fadd_rn(av, red[1][i]);
    }
    const float dtb = __bfloat162float(dt_bias[n]);
    const float al = __bfloat162float(a_log[n]);
    beta[static_cast<long long>(row) * NB + n] = sigmoid_ref(b);
    gate[static_cast<long long>(row) * NB + n] = __fmul_rn(-expf(al), softplus_ref(__fadd_rn(av, dtb)));
  }
}

}  // namespace qlin
