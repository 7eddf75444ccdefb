// Causal prefill attention over the KV cache (kernels/attention.py:136-206).
//
// T new query rows at positions pos0 .. pos0 + T - 1 attend to cache rows
// 0 .. pos0 + t (chunked prefill: earlier chunks are already in the cache).
// The reference's numerics, per key block: K and V are bf16 (an int8 cache
// is dequantised as bf16(code * scale)), S = Q K^T with fp32 accumulation,
// online softmax in fp32, P rounded to bf16 for the P V product, fp32
// accumulation, out = acc / l as bf16.
//
// CTA = 64 query rows of one head (4 warps x 16 rows), key blocks of 32 (the
// reference's block, so the running max that P is rounded against evolves
// the same way).
// Warp-level bf16 MMAs (m16n8k16, fp32 accumulate) on fragments loaded with
// ldmatrix from XOR-swizzled shared memory: Q once per CTA, K and V once per
// key block (V through ldmatrix.trans, so the [key, dim] rows feed the B
// operand directly).  The S accumulator fragments are reused in registers
// as the A fragments of P V.
#pragma once

#include "decode.cuh"
#include "qlin_common.cuh"

namespace qlin {

constexpr int kPaRows = 64;      // query rows per CTA
constexpr int kPaKeys = 32;      // keys per block (the reference's BLOCK_N: P rounds to bf16 against the same running max)
constexpr int kPaThreads = 128;  // 4 warps x 16 query rows

struct AttnPrefillArgs {
  const __nv_bfloat16* q;  // [T, nq * hd], pre-scaled by 1/sqrt(hd)
  const void* kvc;         // [rows, 2 * nkv * hd] bf16 or int8
  const float* kvs;        // [rows, 2 * nkv]
  __nv_bfloat16* out;      // [T, nq * hd]
  int T, pos0, nq, nkv;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

// Byte offset of 16-byte chunk `ch` of row `r` in a tile whose rows hold
// HD bf16 (HD / 8 chunks), chunks XOR-swizzled by the row's low 3 bits.
template <int HD>
__device__ __forceinline__ uint32_t pa_off(int r, int ch) {
  return static_cast<uint32_t>(r * HD * 2 + ((ch ^ (r & 7)) << 4));
}

template <int HD, bool INT8>
__global__ void __launch_bounds__(kPaThreads) attn_prefill_kernel(const __grid_constant__ AttnPrefillArgs a) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t pa_smem[];
  uint8_t* sq = pa_smem;                            // [64][HD] bf16
  uint8_t* sk = sq + kPaRows * HD * 2;              // [kPaKeys][HD] bf16
  uint8_t* sv = sk + kPaKeys * HD * 2;              // [kPaKeys][HD] bf16
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mb = blockIdx.x, head = blockIdx.y;
  const int kvh = head / (a.nq / a.nkv);
  const int sns = 2 * a.nkv;
  const int m0 = mb * kPaRows;
  pdl_wait();
  // Q tile (rows past T are zero)
  for (int i = threadIdx.x; i < kPaRows * CH; i += kPaThreads) {
    const int r = i / CH, ch = i % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m0 + r < a.T)
      v = *reinterpret_cast<const uint4*>(a.q + static_cast<long long>(m0 + r) * a.nq * HD + head * HD + ch * 8);
    *reinterpret_cast<uint4*>(sq + pa_off<HD>(r, ch)) = v;
  }
  const int qend = (m0 + kPaRows < a.T ? m0 + kPaRows : a.T);
  const int nkeys = a.pos0 + qend;  // keys 0 .. pos0 + qend - 1
  const int g = lane >> 2, tig = lane & 3;
  const int row0 = warp * 16 + g, row1 = row0 + 8;        // this thread's two query rows (CTA-local)
  const int qpos0 = a.pos0 + m0 + row0, qpos1 = qpos0 + 8;
  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
  const uint32_t sq_u = smem_u32(sq), sk_u = smem_u32(sk), sv_u = smem_u32(sv);
  for (int n0 = 0; n0 < nkeys; n0 += kPaKeys) {
    __syncthreads();  // the previous block's K / V reads are done (and Q is stored)
    // K and V block -> bf16 tiles (an int8 cache dequantised as bf16(code * scale))
    for (int i = threadIdx.x; i < kPaKeys * CH; i += kPaThreads) {
      const int r = i / CH, ch = i % CH;
      const int n = n0 + r;
      uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
      if (n < nkeys) {
        const long long row = static_cast<long long>(n) * sns * HD;
        if constexpr (INT8) {
          const int8_t* kv = static_cast<const int8_t*>(a.kvc);
          const float ks = a.kvs[static_cast<long long>(n) * sns + kvh];
          const float vs = a.kvs[static_cast<long long>(n) * sns + a.nkv + kvh];
          float kf[8], vf[8];
          load_i8<8>(kv + row + kvh * HD + ch * 8, kf);
          load_i8<8>(kv + row + (a.nkv + kvh) * HD + ch * 8, vf);
          kv4 = make_uint4(pack_bf16x2(__fmul_rn(kf[0], ks), __fmul_rn(kf[1], ks)),
                           pack_bf16x2(__fmul_rn(kf[2], ks), __fmul_rn(kf[3], ks)),
                           pack_bf16x2(__fmul_rn(kf[4], ks), __fmul_rn(kf[5], ks)),
                           pack_bf16x2(__fmul_rn(kf[6], ks), __fmul_rn(kf[7], ks)));
          vv4 = make_uint4(pack_bf16x2(__fmul_rn(vf[0], vs), __fmul_rn(vf[1], vs)),
                           pack_bf16x2(__fmul_rn(vf[2], vs), __fmul_rn(vf[3], vs)),
                           pack_bf16x2(__fmul_rn(vf[4], vs), __fmul_rn(vf[5], vs)),
                           pack_bf16x2(__fmul_rn(vf[6], vs), __fmul_rn(vf[7], vs)));
        } else {
          const __nv_bfloat16* kv = static_cast<const __nv_bfloat16*>(a.kvc);
          kv4 = *reinterpret_cast<const uint4*>(kv + row + kvh * HD + ch * 8);
          vv4 = *reinterpret_cast<const uint4*>(kv + row + (a.nkv + kvh) * HD + ch * 8);
        }
      }
      *reinterpret_cast<uint4*>(sk + pa_off<HD>(r, ch)) = kv4;
      *reinterpret_cast<uint4*>(sv + pa_off<HD>(r, ch)) = vv4;
    }
    __syncthreads();
    // S = Q K^T for this warp's 16 rows x 32 keys (4 tiles of 8 keys)
    constexpr int NT = kPaKeys / 8;
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll 4
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int ch = 2 * kk + (lane >> 4);
        ldsm_x4(sq_u + pa_off<HD>(r, ch), a0, a1, a2, a3);
      }
#pragma unroll
      for (int jp = 0; jp < NT / 2; ++jp) {  // two 8-key tiles per ldmatrix.x4
        uint32_t b0, b1, b2, b3;
        const int r = jp * 16 + (lane & 7) + 8 * (lane >> 4);
        const int ch = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(sk_u + pa_off<HD>(r, ch), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[2 * jp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // causal mask, online softmax (rows row0 / row1; a row's keys are spread
    // over the 4 lanes of a quad)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = n0 + j * 8 + 2 * tig + (e & 1);
        const int qp = e < 2 ? qpos0 : qpos1;
        if (n > qp || n >= nkeys) s[j][e] = -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[j][e]);
      }
    }
    float alpha[2], mnew[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      mnew[h] = fmaxf(mrow[h], mx[h]);
      // a row that has seen no key yet keeps m = -inf: no rescale, p = 0
      alpha[h] = mnew[h] == -INFINITY ? 1.0f : expf(mrow[h] - mnew[h]);
    }
    float psum[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float p = mnew[h] == -INFINITY ? 0.0f : expf(s[j][e] - mnew[h]);
        s[j][e] = p;
        psum[h] = __fadd_rn(psum[h], p);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      psum[h] = __fadd_rn(psum[h], __shfl_xor_sync(0xffffffffu, psum[h], 1));
      psum[h] = __fadd_rn(psum[h], __shfl_xor_sync(0xffffffffu, psum[h], 2));
      lrow[h] = __fadd_rn(__fmul_rn(lrow[h], alpha[h]), psum[h]);
      mrow[h] = mnew[h];
    }
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      o[j][0] = __fmul_rn(o[j][0], alpha[0]);
      o[j][1] = __fmul_rn(o[j][1], alpha[0]);
      o[j][2] = __fmul_rn(o[j][2], alpha[1]);
      o[j][3] = __fmul_rn(o[j][3], alpha[1]);
    }
    // O += P V, P as bf16 A fragments straight from the S accumulators
#pragma unroll
    for (int kk = 0; kk < kPaKeys / 16; ++kk) {
      const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < HD / 16; ++jp) {  // two 8-dim tiles per ldmatrix.x4.trans
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int ch = 2 * jp + (lane >> 4);
        ldsm_x4_t(sv_u + pa_off<HD>(r, ch), b0, b1, b2, b3);
        mma_bf16(o[2 * jp], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * jp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }
  // out = acc / l (rows past T are not stored; l = 0 only for them)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = m0 + (h == 0 ? row0 : row1);
    if (r >= a.T) continue;
    const float inv_l = lrow[h] > 0.0f ? lrow[h] : 1.0f;
    __nv_bfloat16* dst = a.out + static_cast<long long>(r) * a.nq * HD + head * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      const float v0 = __fdiv_rn(o[j][2 * h], inv_l), v1 = __fdiv_rn(o[j][2 * h + 1], inv_l);
      *reinterpret_cast<uint32_t*>(dst + j * 8 + 2 * tig) = pack_bf16x2(v0, v1);
    }
  }
}

__host__ __device__ constexpr int attn_prefill_smem(int HD) { return (kPaRows + 2 * kPaKeys) * HD * 2; }

}  // namespace qlin
