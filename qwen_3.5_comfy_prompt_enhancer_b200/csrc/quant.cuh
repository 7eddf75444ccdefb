// Per-64-group int8 activation quantisation (kernels/norm.py:15-25, 75-92).
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kQuantWarps = 8;

// One warp per (row, 64-element group); lane l owns elements 2l and 2l+1.
//   s = max(amax / 127, 1e-8)           IEEE division, as the reference's fp32 `/`
//   q = round_i8(x / s)                 true division, round half away from zero
__global__ void __launch_bounds__(kQuantWarps * 32) quant_row_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int M, int K, int8_t* __restrict__ q,
    float* __restrict__ s) {
  // The next launch (a projection of these activations) may be placed at
  // once and stream its weights; its own grid-dependency wait still waits for
  // this grid to complete.
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = K / kGroup;
  const int g = blockIdx.x * kQuantWarps + warp;
  const int row = blockIdx.y;
  if (g < G) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(
        x + static_cast<long long>(row) * ldx + g * kGroup + 2 * lane);
    const float a = __bfloat162float(v.x), b = __bfloat162float(v.y);
    float amax = fmaxf(fabsf(a), fabsf(b));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    char2 out;
    out.x = round_i8(__fdiv_rn(a, sc));
    out.y = round_i8(__fdiv_rn(b, sc));
    *reinterpret_cast<char2*>(q + static_cast<long long>(row) * K + g * kGroup + 2 * lane) = out;
    if (lane == 0) s[static_cast<long long>(row) * G + g] = sc;
  }
}

// Same quantisation with 8 elements per lane: one 16-byte load of 8 bf16, the
// group's amax reduced over the 8 lanes that hold its 64 elements, one 8-byte
// store of the codes.  A warp covers 4 groups of one row, a CTA 32 groups.
// For rows of 16-byte aligned x (row stride a multiple of 8) and 8-byte
// aligned q; per element the arithmetic is the kernel's above.
constexpr int kQuantVecGroups = kQuantWarps * 4;  // groups per CTA
__global__ void __launch_bounds__(kQuantWarps * 32) quant_row_vec_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, int M, int K, int8_t* __restrict__ q,
    float* __restrict__ s) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = K / kGroup;
  const int g = blockIdx.x * kQuantVecGroups + warp * 4 + (lane >> 3);
  const int sub = lane & 7;  // 8-element slice of the group
  const int row = blockIdx.y;
  float v[8];
  float amax = 0.0f;
  if (g < G) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<long long>(row) * ldx + g * kGroup + sub * 8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      v[2 * i] = __bfloat162float(b2.x);
      v[2 * i + 1] = __bfloat162float(b2.y);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (g < G) {
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = static_cast<uint8_t>(round_i8(__fdiv_rn(v[i], sc)));
      packed[i >> 2] |= b << (8 * (i & 3));
    }
    *reinterpret_cast<uint2*>(q + static_cast<long long>(row) * K + g * kGroup + sub * 8) =
        make_uint2(packed[0], packed[1]);
    if (sub == 0) s[static_cast<long long>(row) * G + g] = sc;
  }
}

}  // namespace qlin
