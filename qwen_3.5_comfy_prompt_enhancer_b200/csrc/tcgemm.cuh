// Tensor-core GEMM for large M (prefill): W8A8, int8 x int8 -> per-64-K-group
// int32 on tcgen05, promoted to fp32 with the activation row scale of that
// group, exactly as the reference's K loop (kernels/gemm.py:40-52):
//   acc[m, n] += float(sum_{k in group} a_q[m, k] * b[k, n]) * a_s[m, group]
//   out[m, n]  = bf16(acc[m, n] * b_s[n] (+ residual[m, n]))
//
// Tile: 128 activation rows (MMA M = tensor-memory lanes, one row per
// epilogue thread) x 256 output columns, issued as two 128-column halves
// (N = 128 each).  Each half is one 128-column tile of a column segment, so
// proj3's segments (kernels/gemm.py:234-287) need no special case; the fused
// gate/up (kernels/gemm.py:95-231) pairs the gate and up tiles of the same
// columns, and each epilogue thread holds 64 columns of both halves.  A stage
// holds 128 K (two groups): the activation box (K-major, 128-byte swizzle)
// and one weight box per half (the engine's [K, N] rows are MN-major for
// the MMA, 128-byte swizzle).
//
// Promotion cost.  Every group of every output element needs int32 -> fp32
// and a multiply-add.  Each int32 accumulator buffer is pre-filled with the
// bit pattern of 2^23 + 2^22 (0x4B400000) and the MMAs always accumulate, so
// the buffer ends holding 0x4B400000 + I; |I| <= 64 * 128 * 128 < 2^22,
// hence the bits read as the float 12582912 + I exactly, and one
// subtraction recovers float(I) with no conversion instruction.  Two fp32
// lanes per instruction (f32x2) halve the rest.
//
// Warp roles (320 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer over a 4-stage ring
//   warp 1      tensor-memory owner (512 columns = 2 buffers x 256) and MMA issuer
//   warps 2-9   epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows) of
//               half (w-2)/4; per group it loads 128 int32 columns in chunks
//               of 32, writes the magic constant back (re-arming the buffer),
//               and accumulates; at the end of a tile it applies b_s (and the
//               residual) and stores bf16.
#pragma once

#include "args.cuh"
#include "qlin_common.cuh"

namespace qlin {

constexpr int kGmRows = 128;                 // activation rows per tile
constexpr int kGmStages = 4;
constexpr int kGmThreads = 320;
constexpr uint32_t kGmStageA = 128 * 128;    // activation box: 128 K x 128 rows
constexpr uint32_t kGmStageB = 128 * 128;    // weight box per half: 128 columns x 128 K
constexpr uint32_t kGmStageBytes = kGmStageA + 2 * kGmStageB;
constexpr uint32_t kGmMagic = 0x4B400000u;   // bits of 12582912.0f = 2^23 + 2^22
constexpr uint32_t kGmSmem = kGmStages * kGmStageBytes + 256 + 1024;

struct GemmArgs {
  CUtensorMap ta;     // a_q [M, K] int8, box 128 K x 128 rows, 128-byte swizzle
  GemvSeg seg[3];     // W8 column segments; tw box 128 columns x 128 K, 128-byte swizzle
  int nseg;
  int half_tiles;     // 128-column tiles over all segments
  const float* a_s;   // [M, K/64]
  int M, K;
  void* out;          // bf16, row stride ldo (elements)
  long long ldo;
  const void* res;    // bf16 residual or null, row stride ldr
  long long ldr;
  int vec_out;        // 16-byte vector stores / residual loads are aligned
  int8_t* out_q;      // kEpiSiluQuant: int8 [M, n_q]
  float* out_s;       // kEpiSiluQuant: fp32 [M, n_q / 64]
  int n_q;
  unsigned* fault;
};

template <class Args>
__device__ __forceinline__ int gm_seg_of(const Args& p, int ht) {
  int si = 0;
  if (p.nseg > 1 && ht >= p.seg[1].tile_begin) si = 1;
  if (p.nseg > 2 && ht >= p.seg[2].tile_begin) si = 2;
  return si;
}

// Half h of column pair pt: plain projections walk the 128-column tiles of
// their segments two at a time; the fused gate/up pairs gate tile pt (seg 0)
// with up tile pt (seg 1), so one thread can hold both for the same columns.
// HS: 128-column halves per tile -- 2, or 1 for plain outputs whose 256-column
// tiles would leave SMs idle (twice the tiles, each draining one half).
template <int EPI, int HS = 2, class Args>
__device__ __forceinline__ bool gm_half(const Args& p, int pt, int h, int& si, int& n0) {
  if (EPI == kEpiOut) {
    const int ht = HS * pt + h;
    if (h >= HS || ht >= p.half_tiles) return false;
    int s = 0;
    if (p.nseg > 1 && ht >= p.seg[1].tile_begin) s = 1;
    if (p.nseg > 2 && ht >= p.seg[2].tile_begin) s = 2;
    si = s;
    n0 = (ht - p.seg[s].tile_begin) * kTileN;
    return true;
  }
  si = h;
  n0 = pt * kTileN;
  return true;
}

// Fused gate/up epilogue of one row m and the 64 columns [nb, nb + 64): acc
// entries 0..31 hold the gate sums, 32..63 the up sums (two columns each).
// W8 passes its per-column scales (g = acc * sg, u = acc * su,
// kernels/gemm.py:180-197); W4 applied its scales inside the K loop.
//   kEpiSiluBf16:  out[m, n] = bf16(silu(g) * u)
//   kEpiSiluQuant: h = bf16(silu(g) * u); s = max(amax|h| / 127, 1e-8);
//                  q = round_half_away(h / s)   (kernels/gemm.py:198-211)
// The 64 columns are one quantisation group, so the amax stays in-thread.
template <int EPI, class Args>
__device__ __forceinline__ void gm_gate_up_epilogue(const Args& p, int m, int nb, const float2 (&acc)[64],
                                                    const float* sg, const float* su) {
  const int N = p.seg[0].n;
  if (nb >= N) return;
  float hv[64];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int n = nb + 2 * j + e;
      float g = e ? acc[j].y : acc[j].x;
      float u = e ? acc[32 + j].y : acc[32 + j].x;
      if (sg != nullptr && n < N) {
        g = __fmul_rn(g, __ldg(sg + n));
        u = __fmul_rn(u, __ldg(su + n));
      }
      hv[2 * j + e] = __fmul_rn(silu_ref(g), u);
    }
  }
  if constexpr (EPI == kEpiSiluBf16) {
    __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<long long>(m) * p.ldo;
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      const int n = nb + 8 * c8;
      if (n >= N) continue;  // N % 16 == 0
      if (p.vec_out) {
        uint4 ov;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
        for (int e = 0; e < 8; ++e) ob[e] = __float2bfloat16_rn(hv[8 * c8 + e]);
        *reinterpret_cast<uint4*>(orow + n) = ov;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) orow[n + e] = __float2bfloat16_rn(hv[8 * c8 + e]);
      }
    }
  } else {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 64; ++e) {
      hv[e] = bf16_round_f32(hv[e]);
      amax = fmaxf(amax, fabsf(hv[e]));
    }
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    int8_t* qrow = p.out_q + static_cast<long long>(m) * p.n_q + nb;
#pragma unroll
    for (int e = 0; e < 64; ++e) qrow[e] = round_i8(__fdiv_rn(hv[e], sc));
    p.out_s[static_cast<long long>(m) * (p.n_q / 64) + nb / 64] = sc;
  }
}

template <int EPI, int HS>
__global__ void __launch_bounds__(kGmThreads, 1) tc_gemm_kernel(const __grid_constant__ GemmArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGmStages * kGmStageBytes);
  uint64_t* empty = full + kGmStages;
  uint64_t* tfull = empty + kGmStages;   // 2 accumulator buffers
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.K / kGroup;
  const int nstage = (G + 1) / 2;
  const int mtiles = (p.M + kGmRows - 1) / kGmRows;
  const int ptiles = (p.half_tiles + HS - 1) / HS;
  const int tiles = mtiles * ptiles;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < kGmStages; ++i) {
        mbar_init(full + i, 1);
        mbar_init(empty + i, 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(tfull + i, 1);
        mbar_init(tempty + i, 256);
      }
      fence_mbar_init();
    }
    __syncwarp();
  } else if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    uint32_t sc = 0;
    bool ok = true;
    const uint64_t pol_a = l2_policy_evict_last(), pol_b = l2_policy_evict_last();
    for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      const int m0 = (t % mtiles) * kGmRows;
      const int pt = t / mtiles;
      for (int st = 0; st < nstage; ++st, ++sc) {
        const int slot = sc % kGmStages;
        if (!mbar_wait(empty + slot, ((sc / kGmStages) & 1) ^ 1)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          uint8_t* sa = smem + slot * kGmStageBytes;
          uint32_t bytes = kGmStageA;
          for (int h = 0; h < HS; ++h)
            if (HS * pt + h < p.half_tiles) bytes += kGmStageB;
          mbar_arrive_expect_tx(full + slot, bytes);
          tma_load_2d(sa, &p.ta, st * 128, m0, full + slot, pol_a);
          for (int h = 0; h < 2; ++h) {
            int si, n0;
            if (!gm_half<EPI, HS>(p, pt, h, si, n0)) continue;
            tma_load_2d(sa + kGmStageA + h * kGmStageB, &p.seg[si].tw, n0, st * 128, full + slot, pol_b);
          }
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) record_fault(p.fault, kFaultEmptyWait);
    // Copies still in flight land before the CTA may exit.
    const uint32_t issued = sc;
    for (uint32_t i = issued > kGmStages ? issued - kGmStages : 0; i < issued; ++i)
      mbar_wait(full + i % kGmStages, (i / kGmStages) & 1);
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_i8(128, 128, true, true, false, true);
    uint32_t sc = 0, gc = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      const int pt = t / mtiles;
      const int nh = HS == 2 && 2 * pt + 1 < p.half_tiles ? 2 : 1;
      for (int st = 0; ok && st < nstage; ++st, ++sc) {
        const int slot = sc % kGmStages;
        ok = mbar_wait(full + slot, (sc / kGmStages) & 1);
        const int ng = (2 * st + 1 < G) ? 2 : 1;
        for (int gi = 0; ok && gi < ng; ++gi, ++gc) {
          const int b = gc & 1;
          ok = mbar_wait(tempty + b, (gc >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t sa = smem_u32(smem + slot * kGmStageBytes);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t ad = smem_desc(sa + gi * 64 + kk * 32, 16, 1024, kLayoutSw128);
              for (int h = 0; h < nh; ++h) {
                const uint64_t bd =
                    smem_desc(sa + kGmStageA + h * kGmStageB + (gi * 64 + kk * 32) * 128, 8192, 1024, kLayoutSw128);
                tc_mma_i8(tbase + b * 256 + h * 128, ad, bd, idesc, 1u);
              }
            }
            tc_commit(tfull + b);
            if (gi == ng - 1) tc_commit(empty + slot);
          }
          __syncwarp();
        }
      }
    }
    if (!ok && lane == 0) record_fault(p.fault, kFaultMmaWait);
  } else {
    // ------------------------------------------------------------------ epilogue
    // Thread = one row (TMEM lane) x the 64 columns [64c2, 64c2 + 64) of BOTH
    // halves: for the fused gate/up that is the gate and the up value of the
    // same 64 output columns -- one quantisation group, reduced in-thread.
    const int q = warp & 3;          // TMEM lane quarter = rows 32q .. 32q+31
    const int c2 = (warp - 2) >> 2;  // which 64 columns of each half
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(32 * q) << 16) + c2 * 64;
    // Arm both buffers with the magic bits.
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        tmem_fill32(lane_base + b * 256 + hh * 128, kGmMagic);
        tmem_fill32(lane_base + b * 256 + hh * 128 + 32, kGmMagic);
      }
    tc_wait_st();
    tc_fence_before();
    mbar_arrive(tempty + 0);
    mbar_arrive(tempty + 1);

    uint32_t gc = 0;
    bool ok = true;
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      const int m0 = (t % mtiles) * kGmRows;
      const int pt = t / mtiles;
      const int m = m0 + 32 * q + lane;
      const bool mvalid = m < p.M;
      const float* asrow = p.a_s + static_cast<long long>(mvalid ? m : 0) * G;
      float2 acc[64];  // [0, 32): half 0 columns, [32, 64): half 1 columns, two per entry
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = make_float2(0.0f, 0.0f);
      float s_next = mvalid ? __ldg(asrow) : 0.0f;
      for (int g = 0; g < G; ++g, ++gc) {
        const int b = gc & 1;
        const float s = s_next;
        if (g + 1 < G) s_next = mvalid ? __ldg(asrow + g + 1) : 0.0f;
        ok = mbar_wait(tfull + b, (gc >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const float2 s2 = make_float2(s, s);
#pragma unroll
        for (int c = 0; c < 4 * HS; ++c) {
          const uint32_t col = b * 256 + (c >> 2) * 128 + 16 * (c & 3);
          uint32_t r[16];
          tmem_ld32<16>(lane_base + col, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2 v = f2_add(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), neg_magic);
            acc[8 * c + j] = f2_fma(v, s2, acc[8 * c + j]);
          }
          if (c & 1) tmem_fill32(lane_base + col - 16, kGmMagic);  // re-arm the 32 columns just read
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(tempty + b);
      }
      if (!ok) break;
      if (!mvalid) continue;
      // ---------------------------------------------------------------- tile epilogue
      if constexpr (EPI == kEpiOut) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          int si, n0;
          if (!gm_half<EPI, HS>(p, pt, hh, si, n0)) continue;
          const GemvSeg& sg = p.seg[si];
          __nv_bfloat16* orow =
              reinterpret_cast<__nv_bfloat16*>(p.out) + static_cast<long long>(m) * p.ldo + sg.out_col;
          const __nv_bfloat16* rrow =
              p.res ? reinterpret_cast<const __nv_bfloat16*>(p.res) + static_cast<long long>(m) * p.ldr + sg.out_col
                    : nullptr;
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const int n = n0 + c2 * 64 + 8 * c8;
            if (n >= sg.n) continue;  // N % 16 == 0: a chunk of 8 is all in or all out
            float v[8];
            // out * b_s (kernels/gemm.py:51-52); every lane of the warp reads the same scales
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              v[2 * e] = __fmul_rn(acc[32 * hh + 4 * c8 + e].x, __ldg(sg.bs + n + 2 * e));
              v[2 * e + 1] = __fmul_rn(acc[32 * hh + 4 * c8 + e].y, __ldg(sg.bs + n + 2 * e + 1));
            }
            if (rrow) {
              if (p.vec_out) {
                const uint4 rv = *reinterpret_cast<const uint4*>(rrow + n);
                const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], __bfloat162float(rb[e]));
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], __bfloat162float(rrow[n + e]));
              }
            }
            if (p.vec_out) {
              uint4 ov;
              __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
              for (int e = 0; e < 8; ++e) ob[e] = __float2bfloat16_rn(v[e]);
              *reinterpret_cast<uint4*>(orow + n) = ov;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) orow[n + e] = __float2bfloat16_rn(v[e]);
            }
          }
        }
      } else {
        gm_gate_up_epilogue<EPI>(p, m, pt * kTileN + c2 * 64, acc, p.seg[0].bs, p.seg[1].bs);
      }
    }
    if (!ok && lane == 0) record_fault(p.fault, kFaultFullWait);
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace qlin
