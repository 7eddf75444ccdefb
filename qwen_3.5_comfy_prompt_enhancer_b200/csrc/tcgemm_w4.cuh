// Tensor-core GEMM for large M (prefill) with W4 weights: int8 activations x
// group-quantised 4-bit weights, per-(64-K sub-block) int32 on tcgen05,
// promoted exactly as the reference's K loop (kernels/w4.py:64-136):
//   w[k, n]    = nibble(k, n) - z[k / WG, n]          (z = 8 without zeros)
//   acc[m, n] += float(sum_{k in sub-block} a_q[m, k] * w[k, n]) * (a_s[m, k/64] * ws[k / WG, n])
//   out[m, n]  = bf16(acc[m, n] (+ residual[m, n]))
// for weight groups WG that are multiples of 64 (one activation scale and one
// weight scale per 64-K sub-block).  WG = 32 stays on the small-M kernel.
//
// Same tiling, pipeline and promotion as the W8 GEMM (tcgemm.cuh): 128 rows x
// 256 columns per tile (two 128-column halves of the column segments),
// persistent CTAs, int32 group sums in two tensor-memory buffers armed with
// the bits of 2^23 + 2^22.  Differences:
//   * a stage carries the packed nibbles (64 packed rows = 128 K per half),
//     the bf16 scale rows and the zero rows of its groups;
//   * two unpack warps turn each stage into signed int8 tiles (nibble - z,
//     one carry-free byte subtraction per 4 weights) in a 2-slot ring of
//     MN-major 128-byte-swizzled operand tiles, and copy the group scales,
//     converted to fp32, into an 8-slot ring that outlives the raw stage;
//   * the epilogue multiplies the row's activation scale by each column's
//     weight scale before the multiply-add, in the reference's order;
//   * launches with fewer tiles than SMs (column shards of a tensor-parallel
//     layer, mid-size M) cut each tile's K into `kparts` stage ranges, one CTA
//     each.  The parts' fp32 sums meet in a workspace; once every part of the
//     tile has arrived (a counter, a bounded wait -- all CTAs are resident:
//     grid = tiles x kparts <= SMs at one CTA per SM), CTA kp adds the parts
//     of rows [kp x 128 / kparts, ...) in part order and runs the epilogue on
//     them, so the reduction is spread over the tile's CTAs.
#pragma once

#include "tcgemm.cuh"

namespace qlin {

constexpr int kG4Stages = 4;
constexpr int kG4Threads = 384;                 // 12 warps
constexpr int kG4WarpUnpack = 10;               // warps 10, 11
constexpr int kG4UnpackThreads = 64;
constexpr int kG4UBufs = 2;                     // unpacked operand ring (stages)
constexpr int kG4ScaleSlots = 8;                // per-group fp32 scale ring
constexpr uint32_t kG4A = 128 * 128;            // activation box: 128 K x 128 rows
constexpr uint32_t kG4Packed = 64 * 128;        // per half: 64 packed rows x 128 columns
constexpr uint32_t kG4Scale = 2 * 128 * 2;      // per half: up to 2 bf16 scale rows
constexpr uint32_t kG4Zero = 2 * 128;           // per half: up to 2 zero rows
constexpr uint32_t kG4Half = kG4Packed + kG4Scale + kG4Zero;   // 8960, multiple of 128
constexpr uint32_t kG4Stage = kG4A + 2 * kG4Half;                // 34304
constexpr uint32_t kG4StageAligned = (kG4Stage + 1023) / 1024 * 1024;
constexpr uint32_t kG4UTile = 128 * 128;        // unpacked: 128 K rows x 128 columns
constexpr uint32_t kG4UStage = 2 * kG4UTile;
constexpr uint32_t kG4ScaleRing = kG4ScaleSlots * 2 * 128 * 4;   // [slot][half][128] fp32
constexpr uint32_t kG4RawOff = 0;
constexpr uint32_t kG4UOff = kG4Stages * kG4StageAligned;
constexpr uint32_t kG4ScaleOff = kG4UOff + kG4UBufs * kG4UStage;
constexpr uint32_t kG4BarOff = kG4ScaleOff + kG4ScaleRing;
constexpr uint32_t kG4Smem = kG4BarOff + 256 + 1024;
// K parts per tile: at most 16 (128 / kparts >= 8 rows per CTA); the host
// also keeps every part's rows of one CTA (kparts x ceil(128 / kparts) rows
// of HS x 128 fp32) within the stage ring.
constexpr int kG4MaxParts = 16;
static_assert(kG4Smem <= 227 * 1024, "W4 prefill ring exceeds shared memory");

struct GemmW4Args {
  CUtensorMap ta;     // a_q [M, K] int8, box 128 K x 128 rows, 128-byte swizzle
  GemvSeg seg[3];     // tw: packed [K/2, n] box 128 x 64; ts: bf16 [K/WG, n] box 128 x nsr; tz: zeros, same
  int nseg;
  int half_tiles;
  const float* a_s;   // [M, K/64]
  int M, K, wgrp;
  void* out;
  long long ldo;
  const void* res;
  long long ldr;
  int vec_out;
  int8_t* out_q;      // kEpiSiluQuant: int8 [M, n_q]
  float* out_s;       // kEpiSiluQuant: fp32 [M, n_q / 64]
  int n_q;
  int kparts;         // K parts per tile (1: none); > 1 needs grid == tiles * kparts <= SMs
  float* ws;          // kparts > 1: fp32 partial sums [tile][kpart][128 rows][HS * 128]
  unsigned* cnt;      // kparts > 1: per-tile arrival counters, zero at launch
  unsigned* fault;
};

// Scale rows a 128-K stage needs: K/WG rows of the group scale table cover
// [k0, k0 + 128); with WG >= 128 that is one row, with WG = 64 two.
__host__ __device__ constexpr int g4_scale_rows(int wgrp) { return wgrp % 128 == 0 ? 1 : 2; }

__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 x, y, z;\n mov.b64 x, {%2, %3};\n mov.b64 y, {%4, %5};\n mul.rn.f32x2 z, x, y;\n"
      " mov.b64 {%0, %1}, z;\n}\n"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// First stage of K part kp + 1 (the end of part kp) out of `parts` equal
// ranges of `nstage` 128-K stages; kp = -1 gives 0.
__host__ __device__ inline int g4_stage_end(int kp, int parts, int nstage) {
  return static_cast<int>(static_cast<long long>(kp + 1) * nstage / parts);
}

template <int EPI, int HS>
__global__ void __launch_bounds__(kG4Threads, 1) tc_gemm_w4_kernel(const __grid_constant__ GemmW4Args p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kG4BarOff);
  uint64_t* empty = full + kG4Stages;
  uint64_t* ufull = empty + kG4Stages;
  uint64_t* uempty = ufull + kG4UBufs;
  uint64_t* tfull = uempty + kG4UBufs;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);  // (+ the K-part wait flag at [1])
  uint64_t* kbar = tempty + 3;                                       // K-part rows landed
  float* sring = reinterpret_cast<float*>(smem + kG4ScaleOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.K / kGroup;
  const int nstage = (G + 1) / 2;
  const int mtiles = (p.M + kGmRows - 1) / kGmRows;
  const int ptiles = (p.half_tiles + HS - 1) / HS;
  const int tiles = mtiles * ptiles;
  const int units = tiles * p.kparts;  // (tile, K part), tile fastest
  const int nsr = g4_scale_rows(p.wgrp);

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < kG4Stages; ++i) {
        mbar_init(full + i, 1);
        mbar_init(empty + i, 1);
      }
      for (int i = 0; i < kG4UBufs; ++i) {
        mbar_init(ufull + i, kG4UnpackThreads);
        mbar_init(uempty + i, 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(tfull + i, 1);
        mbar_init(tempty + i, 256);
      }
      mbar_init(kbar, 1);
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
    const uint64_t pol = l2_policy_evict_last();
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int t = u % tiles;
      const int m0 = (t % mtiles) * kGmRows;
      const int pt = t / mtiles;
      const int st1 = g4_stage_end(u / tiles, p.kparts, nstage);
      for (int st = g4_stage_end(u / tiles - 1, p.kparts, nstage); st < st1; ++st, ++sc) {
        const int slot = sc % kG4Stages;
        if (!mbar_wait(empty + slot, ((sc / kG4Stages) & 1) ^ 1)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          uint8_t* sa = smem + kG4RawOff + slot * kG4StageAligned;
          uint32_t bytes = kG4A;
          for (int h = 0; h < HS; ++h) {
            int si, n0;
            if (!gm_half<EPI, HS>(p, pt, h, si, n0)) continue;
            bytes += kG4Packed + nsr * 128 * 2 + (p.seg[si].has_z ? nsr * 128 : 0);
          }
          mbar_arrive_expect_tx(full + slot, bytes);
          tma_load_2d(sa, &p.ta, st * 128, m0, full + slot, pol);
          const int srow = (st * 128) / p.wgrp;
          for (int h = 0; h < HS; ++h) {
            int si, n0;
            if (!gm_half<EPI, HS>(p, pt, h, si, n0)) continue;
            const GemvSeg& sg = p.seg[si];
            uint8_t* raw = sa + kG4A + h * kG4Half;
            tma_load_2d(raw, &sg.tw, n0, st * 64, full + slot, pol);
            tma_load_2d(raw + kG4Packed, &sg.ts, n0, srow, full + slot, pol);
            if (sg.has_z) tma_load_2d(raw + kG4Packed + kG4Scale, &sg.tz, n0, srow, full + slot, pol);
          }
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) record_fault(p.fault, kFaultEmptyWait);
    const uint32_t issued = sc;
    for (uint32_t i = issued > kG4Stages ? issued - kG4Stages : 0; i < issued; ++i)
      mbar_wait(full + i % kG4Stages, (i / kG4Stages) & 1);
  } else if (warp >= kG4WarpUnpack) {
    // ------------------------------------------------------------------ unpack
    const int u = threadIdx.x - kG4WarpUnpack * 32;
    uint32_t sc = 0, gbase = 0;
    bool ok = true;
    for (int wu = blockIdx.x; ok && wu < units; wu += gridDim.x) {
      const int pt = (wu % tiles) / mtiles;
      const int st1 = g4_stage_end(wu / tiles, p.kparts, nstage);
      for (int st = g4_stage_end(wu / tiles - 1, p.kparts, nstage); st < st1; ++st, ++sc) {
        const int slot = sc % kG4Stages;
        const int ub = sc % kG4UBufs;
        if (!mbar_wait(full + slot, (sc / kG4Stages) & 1) ||
            !mbar_wait(uempty + ub, ((sc / kG4UBufs) & 1) ^ 1)) {
          ok = false;
          break;
        }
        const int ng = (2 * st + 1 < G) ? 2 : 1;
        const int k0 = st * 128;
        const int srow = k0 / p.wgrp;
        for (int h = 0; h < HS; ++h) {
          int si = 0, n0 = 0;
          const bool valid = gm_half<EPI, HS>(p, pt, h, si, n0);
          const uint8_t* raw = smem + kG4RawOff + slot * kG4StageAligned + kG4A + h * kG4Half;
          uint8_t* ut = smem + kG4UOff + ub * kG4UStage + h * kG4UTile;
          const bool has_z = valid && p.seg[si].has_z;
          // 64 packed rows x 8 chunks of 16 columns; packed row j holds K = 2j
          // (low nibble) and 2j + 1 (high nibble) of 16 columns.
          // All eight chunks are loaded before any is converted and stored, so
          // their shared-memory latencies overlap.
          uint4 vv[8], zz[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int idx = u + kG4UnpackThreads * i;
            const int pr = idx >> 3, ch = idx & 7;
            vv[i] = *reinterpret_cast<const uint4*>(raw + pr * 128 + ch * 16);
            const int zr = (k0 + 2 * pr) / p.wgrp - srow;
            zz[i] = has_z ? *reinterpret_cast<const uint4*>(raw + kG4Packed + kG4Scale + zr * 128 + ch * 16)
                          : make_uint4(0x08080808u, 0x08080808u, 0x08080808u, 0x08080808u);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int idx = u + kG4UnpackThreads * i;
            const int pr = idx >> 3, ch = idx & 7;
            const uint4 v = vv[i], z = zz[i];
            uint4 lo, hi;
            // nibble - z per byte as (nibble + (0x80 - z)) ^ 0x80: no carry
            // or borrow crosses a byte (nibble, z <= 15), same bytes as __vsub4
            const uint4 zc = make_uint4(0x80808080u - z.x, 0x80808080u - z.y, 0x80808080u - z.z, 0x80808080u - z.w);
            lo.x = ((v.x & 0x0F0F0F0Fu) + zc.x) ^ 0x80808080u; hi.x = (((v.x >> 4) & 0x0F0F0F0Fu) + zc.x) ^ 0x80808080u;
            lo.y = ((v.y & 0x0F0F0F0Fu) + zc.y) ^ 0x80808080u; hi.y = (((v.y >> 4) & 0x0F0F0F0Fu) + zc.y) ^ 0x80808080u;
            lo.z = ((v.z & 0x0F0F0F0Fu) + zc.z) ^ 0x80808080u; hi.z = (((v.z >> 4) & 0x0F0F0F0Fu) + zc.z) ^ 0x80808080u;
            lo.w = ((v.w & 0x0F0F0F0Fu) + zc.w) ^ 0x80808080u; hi.w = (((v.w >> 4) & 0x0F0F0F0Fu) + zc.w) ^ 0x80808080u;
            const int r0 = 2 * pr, r1 = 2 * pr + 1;
            *reinterpret_cast<uint4*>(ut + r0 * 128 + ((ch ^ (r0 & 7)) << 4)) = lo;
            *reinterpret_cast<uint4*>(ut + r1 * 128 + ((ch ^ (r1 & 7)) << 4)) = hi;
          }
          // fp32 weight scales of the stage's groups into the ring (two columns per thread)
          const uint16_t* sc16 = reinterpret_cast<const uint16_t*>(raw + kG4Packed);
          for (int gi = 0; gi < ng; ++gi) {
            const int row = (k0 + gi * 64) / p.wgrp - srow;
            float* dst = sring + (((gbase + gi) % kG4ScaleSlots) * 2 + h) * 128;
            dst[2 * u] = bf16_bits_to_f32(sc16[row * 128 + 2 * u]);
            dst[2 * u + 1] = bf16_bits_to_f32(sc16[row * 128 + 2 * u + 1]);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(ufull + ub);
        gbase += ng;
      }
    }
    if (!ok && lane == 0) record_fault(p.fault, kFaultFullWait);
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_i8(128, 128, true, true, false, true);
    uint32_t sc = 0, gc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int pt = (u % tiles) / mtiles;
      const int nh = HS == 2 && 2 * pt + 1 < p.half_tiles ? 2 : 1;
      const int st1 = g4_stage_end(u / tiles, p.kparts, nstage);
      for (int st = g4_stage_end(u / tiles - 1, p.kparts, nstage); ok && st < st1; ++st, ++sc) {
        const int slot = sc % kG4Stages;
        const int ub = sc % kG4UBufs;
        ok = mbar_wait(full + slot, (sc / kG4Stages) & 1) && mbar_wait(ufull + ub, (sc / kG4UBufs) & 1);
        const int ng = (2 * st + 1 < G) ? 2 : 1;
        for (int gi = 0; ok && gi < ng; ++gi, ++gc) {
          const int b = gc & 1;
          ok = mbar_wait(tempty + b, (gc >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t sa = smem_u32(smem + kG4RawOff + slot * kG4StageAligned);
            const uint32_t su = smem_u32(smem + kG4UOff + ub * kG4UStage);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t ad = smem_desc(sa + gi * 64 + kk * 32, 16, 1024, kLayoutSw128);
              for (int h = 0; h < nh; ++h) {
                const uint64_t bd = smem_desc(su + h * kG4UTile + (gi * 64 + kk * 32) * 128, 8192, 1024, kLayoutSw128);
                tc_mma_i8(tbase + b * 256 + h * 128, ad, bd, idesc, 1u);
              }
            }
            tc_commit(tfull + b);
            if (gi == ng - 1) {
              tc_commit(empty + slot);
              tc_commit(uempty + ub);
            }
          }
          __syncwarp();
        }
      }
    }
    if (!ok && lane == 0) record_fault(p.fault, kFaultMmaWait);
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-9)
    // Thread = one row (TMEM lane) x the 64 columns [64c2, 64c2 + 64) of both
    // halves (gate and up of the same columns for the fused epilogue).
    const int q = warp & 3;          // TMEM lane quarter = rows 32q .. 32q+31
    const int c2 = (warp - 2) >> 2;  // which 64 columns of each half
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(32 * q) << 16) + c2 * 64;
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

    // tile epilogue of row m, columns [64 c2e, 64 c2e + 64) of each half, from a
    auto emit = [&](int m, int pt, int c2e, const float2 (&a)[64]) {
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
            const int n = n0 + c2e * 64 + 8 * c8;
            if (n >= sg.n) continue;  // N % 16 == 0: a chunk of 8 is all in or all out
            float v[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              v[2 * e] = a[32 * hh + 4 * c8 + e].x;
              v[2 * e + 1] = a[32 * hh + 4 * c8 + e].y;
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
        gm_gate_up_epilogue<EPI>(p, m, pt * kTileN + c2e * 64, a, nullptr, nullptr);
      }
    };

    uint32_t gc = 0;
    bool ok = true;
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      const int t = u % tiles, kp = u / tiles;
      const int gb = 2 * g4_stage_end(kp - 1, p.kparts, nstage);
      const int ge = min(2 * g4_stage_end(kp, p.kparts, nstage), G);
      const int m0 = (t % mtiles) * kGmRows;
      const int pt = t / mtiles;
      const int m = m0 + 32 * q + lane;
      const bool mvalid = m < p.M;
      int m_e = m, c2_e = c2;  // the row and columns this thread's epilogue writes
      const float* asrow = p.a_s + static_cast<long long>(mvalid ? m : 0) * G;
      float2 acc[64];  // [0, 32): half 0 columns, [32, 64): half 1 columns, two per entry
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = make_float2(0.0f, 0.0f);
      float s_next = mvalid ? __ldg(asrow + gb) : 0.0f;
      for (int g = gb; g < ge; ++g, ++gc) {
        const int b = gc & 1;
        const float as = s_next;
        if (g + 1 < ge) s_next = mvalid ? __ldg(asrow + g + 1) : 0.0f;
        ok = mbar_wait(tfull + b, (gc >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const float2 as2 = make_float2(as, as);
        const float* wsg = sring + (gc % kG4ScaleSlots) * 2 * 128 + c2 * 64;
#pragma unroll
        for (int c = 0; c < 4 * HS; ++c) {
          const int hh = c >> 2;
          const uint32_t col = b * 256 + hh * 128 + 16 * (c & 3);
          uint32_t r[16];
          tmem_ld32<16>(lane_base + col, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            // (a_s * ws) first, then the int32 sum times that (kernels/w4.py:103-104)
            const float2 ws = *reinterpret_cast<const float2*>(wsg + hh * 128 + 16 * (c & 3) + 2 * j);
            const float2 t2 = f2_mul(as2, ws);
            const float2 v = f2_add(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), neg_magic);
            acc[8 * c + j] = f2_fma(v, t2, acc[8 * c + j]);
          }
          if (c & 1) tmem_fill32(lane_base + col - 16, kGmMagic);
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(tempty + b);
      }
      if (!ok) break;
      if (p.kparts > 1) {
        // ---------------------------------------------------------------- K parts of the tile meet
        // (this CTA's only unit: the host launches one CTA per (tile, part))
        const int KP = p.kparts;
        constexpr int RW = HS * 128;  // floats per row of a part
        const int et = threadIdx.x - 64;  // epilogue thread 0..255
        float* wt = p.ws + static_cast<size_t>(t) * KP * 128 * RW;
        float* mine = wt + (static_cast<size_t>(kp) * 128 + 32 * q + lane) * RW + c2 * 64;
#pragma unroll
        for (int c = 0; c < 4 * HS; ++c) {
          float4* d = reinterpret_cast<float4*>(mine + (c >> 2) * 128 + 16 * (c & 3));
#pragma unroll
          for (int e = 0; e < 4; ++e)
            __stcg(d + e, make_float4(acc[8 * c + 2 * e].x, acc[8 * c + 2 * e].y, acc[8 * c + 2 * e + 1].x,
                                      acc[8 * c + 2 * e + 1].y));
        }
        __threadfence();
        named_bar_sync(1, 256);
        volatile int* ks_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
        if (et == 0) {
          atomicAdd(p.cnt + t, 1u);
          const unsigned long long t0 = global_ns();
          int f = 0;
          while (*reinterpret_cast<volatile unsigned*>(p.cnt + t) < static_cast<unsigned>(KP)) {
            if (global_ns() - t0 > wait_limit_ns()) {
              f = 1;
              break;
            }
          }
          *ks_flag = f;
        }
        named_bar_sync(1, 256);
        if (*ks_flag) {
          ok = false;
          break;
        }
        __threadfence();
        // rows [r0, r1) of every part, one bulk copy each, over the stage ring
        // (free: every stage of this unit has been consumed)
        const int r0 = kp * 128 / KP, r1 = (kp + 1) * 128 / KP, nr = r1 - r0;
        const uint32_t slab = static_cast<uint32_t>(nr * RW * 4);
        float* sl = reinterpret_cast<float*>(smem + kG4RawOff);
        if (et == 0) {
          fence_proxy_async_global();
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(kbar, KP * slab);
          for (int k = 0; k < KP; ++k)
            bulk_load(sl + static_cast<size_t>(k) * nr * RW, wt + (static_cast<size_t>(k) * 128 + r0) * RW, slab, kbar);
        }
        if (!mbar_wait(kbar, 0)) {
          if (lane == 0) record_fault(p.fault, kFaultFullWait);
          mbar_wait(kbar, 0);  // the copies land before the region is reused or the CTA exits
          ok = false;
          break;
        }
        // parts added in K order, in place over part 0's rows
        float4* sl4 = reinterpret_cast<float4*>(sl);
        const int n4 = nr * RW / 4;
        for (int x = et; x < n4; x += 256) {
          float4 v = sl4[x];
          for (int k = 1; k < KP; ++k) {
            const float4 w = sl4[k * n4 + x];
            v.x = __fadd_rn(v.x, w.x);
            v.y = __fadd_rn(v.y, w.y);
            v.z = __fadd_rn(v.z, w.z);
            v.w = __fadd_rn(v.w, w.w);
          }
          sl4[x] = v;
        }
        named_bar_sync(1, 256);
        // thread (row r0 + rl, columns c2e) runs the epilogue on the sum
        if (et >= 2 * nr) continue;
        const int rl = et >> 1;
        c2_e = et & 1;
        m_e = m0 + r0 + rl;
        const float* row = sl + rl * RW + c2_e * 64;
#pragma unroll
        for (int c = 0; c < 4 * HS; ++c)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            acc[8 * c + j] = *reinterpret_cast<const float2*>(row + (c >> 2) * 128 + 16 * (c & 3) + 2 * j);
      }
      if (m_e >= p.M) continue;
      emit(m_e, pt, c2_e, acc);
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
