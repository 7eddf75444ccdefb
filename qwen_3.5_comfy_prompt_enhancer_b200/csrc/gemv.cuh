// Decode-side (small M) quantised GEMV family for sm_100a.
//
// One kernel template covers every hot-path entry point when the activation
// has few rows (decode: M = 1..8):
//   kEpiOut        gemm_i8 / gemm_w4 (+ residual) and proj3 / proj3_w4 (up to
//                  three column segments written side by side)
//   kEpiSiluBf16   mlp_gate_up        (two weight streams, bf16 h)
//   kEpiSiluQuant  mlp_gate_up_quant  / mlp_gate_up_quant_w4 (two weight
//                  streams, h rounded through bf16 and re-quantised per 64
//                  columns)
//
// Work decomposition.  The output columns are cut into 128-column tiles
// (128 bytes of one weight row: 128 int8 columns, or 128 packed W4 columns
// holding two K values each).  The K axis is cut into `split` contiguous
// ranges of whole 64-element activation groups; the CTAs that share a tile
// form one thread-block cluster and combine their fp32 partial sums through
// distributed shared memory (no global scratch, fixed summation order).
//
// Inside a CTA one producer warp streams the tile's weight rows (and W4
// group scales / zeros) with 2-D TMA loads into a ring of shared-memory
// stages, one stage per 64-row activation group.  Eight consumer warps own
// the ring slots round-robin; in a warp each lane owns 4 adjacent columns and runs
// over all 64 K rows of the group, so the int32 sum of every
// (row, column, group) is formed completely inside one thread -- exactly the
// reference's per-64-block `tl.dot` (kernels/gemm.py:43, kernels/w4.py:89)
// -- before the fp32 scaling.  Four weight rows are transposed in registers
// with byte permutes so that `dp4a` can reduce along K.
//
// W4 nibbles are never expanded in memory: after the transpose, the low
// nibbles of a 32-bit word are four even-K weights and the high nibbles four
// odd-K weights, and `dp4a.u32.s32` multiplies them (unsigned 0..15) with
// activations pre-split into even/odd K words.  The zero point is folded in
// exactly in integers: sum(a * (nib - z)) = sum(a * nib) - z * sum(a).
//
// PDL: the producer starts streaming weights before `griddepcontrol.wait`
// (weights never depend on the preceding kernel); activations, residuals
// and all outputs are touched only after it.
#pragma once

#include <cooperative_groups.h>

#include "qlin_common.cuh"

namespace qlin {

constexpr int kTileN = 128;
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads + 32;

enum GemvEpi : int { kEpiOut = 0, kEpiSiluBf16 = 1, kEpiSiluQuant = 2 };

struct GemvSeg {
  CUtensorMap tw;    // W8: int8 [K, N]; W4: packed uint8 [K/2, N]
  CUtensorMap ts;    // W4: bf16 group scales [K/WG, N]
  CUtensorMap tz;    // W4: uint8 group zeros [K/WG, N]
  const float* bs;   // W8: fp32 per-column scales [N]
  int n;             // columns in this segment
  int out_col;       // first output column of this segment
  int tile_begin;    // first tile index of this segment
  int has_z;         // W4: zeros present
  const void* w;     // weight base (host side: the prefill paths build their own tensor maps)
  const void* sp;    // W4 scale base (host side)
  const void* zp;    // W4 zero base or null (host side)
};

struct GemvArgs {
  CUtensorMap ta;    // tcgen05 path: activations a_q [M, K], 128-byte-swizzled boxes of 128 K x rows
  GemvSeg seg[3];    // kEpiOut: column segments; gate/up epilogues: seg[0]=gate, seg[1]=up
  int nseg;
  const int8_t* a_q;  // [M, K]
  const float* a_s;   // [M, K/64]
  int M, K, wgrp;
  int split;          // K ranges per tile == cluster size
  int ring;           // stages in the shared-memory ring
  int aring;          // (unused by tc_gemv)
  int bs;             // tc_gemv: 64-K groups per batch (one barrier / commit per batch)
  int rb;             // tc_gemv: batch slots in the weight ring
  int ab;             // tc_gemv W4: batch slots in the unpacked-weight ring
  int nbb;            // tc_gemv: batch accumulators in tensor memory
  int gmax;           // max groups one CTA handles
  int part_alias;     // tc_gemv: partial sums land in rank 0's (finished) MMA operand region
  void* out;          // bf16, row stride ldo
  long long ldo;
  const void* res;    // bf16 residual or null, row stride ldr
  long long ldr;
  int8_t* out_q;      // kEpiSiluQuant: int8 [M, n_q]
  float* out_s;       // kEpiSiluQuant: fp32 [M, n_q/64]
  int n_q;
  unsigned* fault;    // device fault word (bounded waits)
};

struct GemvLayout {
  uint32_t wbytes, sbytes, zbytes, stream_bytes, stage_bytes, ring_bytes;
  uint32_t bar_off, act_off, asum_off, as_off, part_off, xchg_off, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

// Shared-memory carve-up; host and device call this with the same arguments.
__host__ __device__ inline GemvLayout gemv_layout(int wb, int mr, int nstream, int wgrp, int gmax,
                                                  int ring) {
  GemvLayout L;
  const int nsr = (wb == 4 && wgrp == 32) ? 2 : 1;
  L.wbytes = wb == 8 ? 64 * kTileN : 32 * kTileN;
  L.sbytes = wb == 4 ? nsr * kTileN * 2 : 0;
  L.zbytes = wb == 4 ? nsr * kTileN : 0;
  L.stream_bytes = L.wbytes + L.sbytes + L.zbytes;
  L.stage_bytes = nstream * L.stream_bytes;
  const uint32_t red = kConsumerWarps * nstream * mr * kTileN * 4;
  L.ring_bytes = align_up(ring * L.stage_bytes > red ? ring * L.stage_bytes : red, 128);
  uint32_t off = L.ring_bytes;
  L.bar_off = off;
  off = align_up(off + 2 * ring * 8, 16);
  L.act_off = off;
  off = align_up(off + gmax * 64 * mr, 16);
  L.asum_off = off;
  off = align_up(off + (wb == 4 ? gmax * 2 * mr * 4 : 0), 16);
  L.as_off = off;
  off = align_up(off + gmax * mr * 4, 16);
  L.part_off = off;
  off = align_up(off + nstream * mr * kTileN * 4, 16);
  L.xchg_off = off;
  off = align_up(off + 4 * mr * 4, 16);
  L.total = off;
  return L;
}

// ---------------------------------------------------------------------------
// Stage processing: one 64-row activation group of one weight stream.
// ---------------------------------------------------------------------------

template <int MR>
__device__ __forceinline__ void load_act_words(const int* p, int (&aw)[MR]) {
  if constexpr (MR % 4 == 0) {
#pragma unroll
    for (int m = 0; m < MR; m += 4) {
      const int4 v = *reinterpret_cast<const int4*>(p + m);
      aw[m] = v.x; aw[m + 1] = v.y; aw[m + 2] = v.z; aw[m + 3] = v.w;
    }
  } else if constexpr (MR == 2) {
    const int2 v = *reinterpret_cast<const int2*>(p);
    aw[0] = v.x; aw[1] = v.y;
  } else {
#pragma unroll
    for (int m = 0; m < MR; ++m) aw[m] = p[m];
  }
}

// W8: stage = int8 [64][128]; act = int32 words [16][MR] (4 consecutive K each).
template <int MR>
__device__ __forceinline__ void w8_group(const uint8_t* __restrict__ st, const int* __restrict__ act,
                                         const float* __restrict__ asc, int lane,
                                         float (&acc)[MR][4]) {
  int isum[MR][4];
#pragma unroll
  for (int m = 0; m < MR; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) isum[m][j] = 0;
  const uint8_t* w = st + lane * 4;
#pragma unroll 4
  for (int q = 0; q < 16; ++q) {
    const uint32_t r0 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 0) * kTileN);
    const uint32_t r1 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 1) * kTileN);
    const uint32_t r2 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 2) * kTileN);
    const uint32_t r3 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 3) * kTileN);
    uint32_t c[4];
    transpose4x4(r0, r1, r2, r3, c[0], c[1], c[2], c[3]);
    int aw[MR];
    load_act_words<MR>(act + q * MR, aw);
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j) isum[m][j] = dp4a_ss(static_cast<int>(c[j]), aw[m], isum[m][j]);
  }
  // out += float(int32 block sum) * a_s[m, kb]   (kernels/gemm.py:43-45)
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const float s = asc[m];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc[m][j] = __fadd_rn(acc[m][j], __fmul_rn(__int2float_rn(isum[m][j]), s));
  }
}

// W4: stage = packed uint8 [32][128], bf16 scales [nsr][128], uint8 zeros
// [nsr][128]; act = [8 chunks][MR][even word, odd word]; asum = int32
// [2][MR] sums of a over each 32-K half of the group.
template <int MR>
__device__ __forceinline__ void w4_group(const uint8_t* __restrict__ st, uint32_t wbytes,
                                         uint32_t sbytes, int wgrp, int has_z,
                                         const int* __restrict__ act, const int* __restrict__ asum,
                                         const float* __restrict__ asc, int lane,
                                         float (&acc)[MR][4]) {
  const uint8_t* w = st + lane * 4;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + wbytes);
  const uint8_t* zz = st + wbytes + sbytes;
  const int nsub = (wgrp == 32) ? 2 : 1;  // SUB = min(WG, 64) (kernels/w4.py:113)
  const int qper = 8 / nsub;
  for (int sb = 0; sb < nsub; ++sb) {
    int isum[MR][4];
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j) isum[m][j] = 0;
#pragma unroll 4
    for (int qq = 0; qq < qper; ++qq) {
      const int q = sb * qper + qq;
      const uint32_t r0 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 0) * kTileN);
      const uint32_t r1 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 1) * kTileN);
      const uint32_t r2 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 2) * kTileN);
      const uint32_t r3 = *reinterpret_cast<const uint32_t*>(w + (4 * q + 3) * kTileN);
      uint32_t t[4];
      transpose4x4(r0, r1, r2, r3, t[0], t[1], t[2], t[3]);
      int aw[2 * MR];
      load_act_words<2 * MR>(act + q * 2 * MR, aw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo = t[j] & 0x0F0F0F0Fu;          // even K of the 8-K chunk
        const uint32_t hi = (t[j] >> 4) & 0x0F0F0F0Fu;   // odd K
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          isum[m][j] = dp4a_us(lo, aw[2 * m], isum[m][j]);
          isum[m][j] = dp4a_us(hi, aw[2 * m + 1], isum[m][j]);
        }
      }
    }
    // Exact zero-point fold, then out += float(acc) * (a_s * ws)  (kernels/w4.py:84-104)
    uint32_t zw = 0x08080808u;
    if (has_z) zw = *reinterpret_cast<const uint32_t*>(zz + sb * kTileN + lane * 4);
    const uint2 sw = *reinterpret_cast<const uint2*>(sc + sb * kTileN + lane * 4);
    float ws[4];
    ws[0] = bf16_bits_to_f32(static_cast<uint16_t>(sw.x & 0xFFFFu));
    ws[1] = bf16_bits_to_f32(static_cast<uint16_t>(sw.x >> 16));
    ws[2] = bf16_bits_to_f32(static_cast<uint16_t>(sw.y & 0xFFFFu));
    ws[3] = bf16_bits_to_f32(static_cast<uint16_t>(sw.y >> 16));
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const int sa = nsub == 2 ? asum[sb * MR + m] : asum[m] + asum[MR + m];
      const float a = asc[m];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int z = static_cast<int>((zw >> (8 * j)) & 0xFFu);
        const int v = isum[m][j] - z * sa;
        const float t = __fmul_rn(a, ws[j]);
        acc[m][j] = __fadd_rn(acc[m][j], __fmul_rn(__int2float_rn(v), t));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int WB, int MR, int EPI>
__global__ void __launch_bounds__(kGemvThreads, (MR <= 4 ? 2 : 1)) gemv_kernel(const __grid_constant__ GemvArgs p) {
  namespace cg = cooperative_groups;
  constexpr int NS = (EPI == kEpiOut) ? 1 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvLayout L = gemv_layout(WB, MR, NS, p.wgrp, p.gmax, p.ring);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + p.ring;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = blockIdx.x;  // cluster = (split, 1, 1) and gridDim.x == split
  const int tile = blockIdx.y;
  const int m0 = blockIdx.z * MR;

  int si = 0;
  if (EPI == kEpiOut) {
    if (p.nseg > 1 && tile >= p.seg[1].tile_begin) si = 1;
    if (p.nseg > 2 && tile >= p.seg[2].tile_begin) si = 2;
  }
  const GemvSeg& S0 = p.seg[si];
  const int n0 = (tile - S0.tile_begin) * kTileN;
  const int G = p.K / kGroup;
  const int g0 = static_cast<int>(static_cast<long long>(rank) * G / p.split);
  const int g1 = static_cast<int>(static_cast<long long>(rank + 1) * G / p.split);
  const int nst = g1 - g0;

  // Epilogue operands, fetched early by the epilogue threads (rank 0,
  // threads 0..127) so that no global round trip is left after the K loop:
  // W8 column scales now (weights never depend on the preceding kernel), the
  // residual right after the grid-dependency wait.
  const bool epi_thread = (rank == 0) && (threadIdx.x < kTileN);
  const int en = n0 + static_cast<int>(threadIdx.x);
  const bool evalid = epi_thread && en < S0.n;
  float pre_s0 = 1.0f, pre_s1 = 1.0f;
  if (WB == 8 && evalid) {
    pre_s0 = __ldg((NS == 1 ? S0.bs : p.seg[0].bs) + en);
    if (NS == 2) pre_s1 = __ldg(p.seg[1].bs + en);
  }
  float pre_res[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) pre_res[m] = 0.0f;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.ring; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  float* part = reinterpret_cast<float*>(smem + L.part_off);  // [NS][MR][128]

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t bytes = 0;
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        const GemvSeg& sg = NS == 1 ? S0 : p.seg[s];
        bytes += L.wbytes;
        if (WB == 4) bytes += L.sbytes + (sg.has_z ? L.zbytes : 0);
      }
      for (int i = 0; i < nst; ++i) {
        const int slot = i % p.ring;
        if (i >= p.ring && !mbar_wait(empty + slot, ((i / p.ring) - 1) & 1)) {
          atomicOr(p.fault, kFaultEmptyWait);
          break;
        }
        mbar_arrive_expect_tx(full + slot, bytes);
        const int g = g0 + i;
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const GemvSeg& sg = NS == 1 ? S0 : p.seg[s];
          uint8_t* dst = smem + slot * L.stage_bytes + s * L.stream_bytes;
          tma_load_2d(dst, &sg.tw, n0, WB == 8 ? g * 64 : g * 32, full + slot, pol);
          if (WB == 4) {
            const int srow = (g * 64) / p.wgrp;
            tma_load_2d(dst + L.wbytes, &sg.ts, n0, srow, full + slot, pol);
            if (sg.has_z) tma_load_2d(dst + L.wbytes + L.sbytes, &sg.tz, n0, srow, full + slot, pol);
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ consumers
    pdl_wait();
    const int tid = threadIdx.x;
    if (EPI == kEpiOut && evalid && p.res) {
      const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(p.res);
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m0 + m < p.M)
          pre_res[m] = __bfloat162float(res[static_cast<long long>(m0 + m) * p.ldr + S0.out_col + en]);
    }
    int* actw = reinterpret_cast<int*>(smem + L.act_off);
    int* asum = reinterpret_cast<int*>(smem + L.asum_off);
    float* ass = reinterpret_cast<float*>(smem + L.as_off);
    const int kbase = g0 * 64;
    if (WB == 8) {
      // words [kq][MR]: 16-byte chunks of each row's K range
      const int nch = nst * 4;
      for (int idx = tid; idx < MR * nch; idx += kConsumerThreads) {
        const int m = idx / nch, ch = idx - m * nch;
        int4 v = make_int4(0, 0, 0, 0);
        if (m0 + m < p.M)
          v = __ldg(reinterpret_cast<const int4*>(p.a_q + static_cast<long long>(m0 + m) * p.K +
                                                   kbase + ch * 16));
        actw[(ch * 4 + 0) * MR + m] = v.x;
        actw[(ch * 4 + 1) * MR + m] = v.y;
        actw[(ch * 4 + 2) * MR + m] = v.z;
        actw[(ch * 4 + 3) * MR + m] = v.w;
      }
    } else {
      // [k8][MR][even, odd] words + per-32-K sums of a
      const int nch = nst * 2;  // 32-byte chunks
      for (int idx = tid; idx < MR * nch; idx += kConsumerThreads) {
        const int m = idx / nch, ch = idx - m * nch;
        int4 v0 = make_int4(0, 0, 0, 0), v1 = make_int4(0, 0, 0, 0);
        if (m0 + m < p.M) {
          const int4* src = reinterpret_cast<const int4*>(
              p.a_q + static_cast<long long>(m0 + m) * p.K + kbase + ch * 32);
          v0 = __ldg(src);
          v1 = __ldg(src + 1);
        }
        const uint32_t w[8] = {(uint32_t)v0.x, (uint32_t)v0.y, (uint32_t)v0.z, (uint32_t)v0.w,
                               (uint32_t)v1.x, (uint32_t)v1.y, (uint32_t)v1.z, (uint32_t)v1.w};
        int s = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int k8 = ch * 4 + c;
          actw[(k8 * MR + m) * 2 + 0] = static_cast<int>(__byte_perm(w[2 * c], w[2 * c + 1], 0x6420));
          actw[(k8 * MR + m) * 2 + 1] = static_cast<int>(__byte_perm(w[2 * c], w[2 * c + 1], 0x7531));
          s = dp4a_ss(static_cast<int>(w[2 * c]), 0x01010101, s);
          s = dp4a_ss(static_cast<int>(w[2 * c + 1]), 0x01010101, s);
        }
        asum[ch * MR + m] = s;
      }
    }
    for (int idx = tid; idx < MR * nst; idx += kConsumerThreads) {
      const int m = idx / nst, gl = idx - m * nst;
      ass[gl * MR + m] = (m0 + m < p.M) ? __ldg(p.a_s + static_cast<long long>(m0 + m) * G + g0 + gl) : 0.0f;
    }
    named_bar_sync(1, kConsumerThreads);
    pdl_launch_dependents();

    float acc[NS][MR][4];
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[s][m][j] = 0.0f;

    // Ring slot s is always consumed by warp s % kConsumerWarps, so every slot's
    // fills are waited for in order by one warp (an mbarrier parity wait is
    // only unambiguous when the previous phase has been observed).
    for (int i = 0; i < nst; ++i) {
      const int slot = i % p.ring;
      if (slot % kConsumerWarps != warp) continue;
      if (!mbar_wait(full + slot, (i / p.ring) & 1)) {
        if (lane == 0) atomicOr(p.fault, kFaultFullWait);
        break;
      }
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        const uint8_t* st = smem + slot * L.stage_bytes + s * L.stream_bytes;
        if (WB == 8) {
          w8_group<MR>(st, actw + i * 16 * MR, ass + i * MR, lane, acc[s]);
        } else {
          const GemvSeg& sg = NS == 1 ? S0 : p.seg[s];
          w4_group<MR>(st, L.wbytes, L.sbytes, p.wgrp, sg.has_z, actw + i * 16 * MR,
                       asum + i * 2 * MR, ass + i * MR, lane, acc[s]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + slot);
    }

    // Cross-warp reduction in a fixed order, through the (now idle) ring.
    named_bar_sync(1, kConsumerThreads);
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m)
        *reinterpret_cast<float4*>(red + ((warp * NS + s) * MR + m) * kTileN + lane * 4) =
            make_float4(acc[s][m][0], acc[s][m][1], acc[s][m][2], acc[s][m][3]);
    named_bar_sync(1, kConsumerThreads);
    for (int idx = tid; idx < NS * MR * kTileN; idx += kConsumerThreads) {
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) v = __fadd_rn(v, red[w * NS * MR * kTileN + idx]);
      part[idx] = v;
    }
  }

  // ------------------------------------------------------------ cluster combine + epilogue
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (rank == 0 && threadIdx.x < kTileN) {
    const int c = threadIdx.x;
    const int n = n0 + c;
    const bool valid = n < S0.n;
    float vs[NS][MR];
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m) vs[s][m] = 0.0f;
    for (int r = 0; r < p.split; ++r) {
      const float* rp = cluster.map_shared_rank(part, r);
#pragma unroll
      for (int s = 0; s < NS; ++s)
#pragma unroll
        for (int m = 0; m < MR; ++m) vs[s][m] = __fadd_rn(vs[s][m], rp[(s * MR + m) * kTileN + c]);
    }
    if (EPI == kEpiOut) {
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (!valid || m0 + m >= p.M) continue;
        float v = vs[0][m];
        if (WB == 8) v = __fmul_rn(v, pre_s0);  // out * bs (kernels/gemm.py:51-52)
        if (p.res) v = __fadd_rn(v, pre_res[m]);
        out[static_cast<long long>(m0 + m) * p.ldo + S0.out_col + n] = __float2bfloat16_rn(v);
      }
    } else {
      const float sg = pre_s0, su = pre_s1;
      float* xchg = reinterpret_cast<float*>(smem + L.xchg_off);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float g = vs[0][m], u = vs[1][m];
        if (WB == 8) {
          g = __fmul_rn(g, sg);
          u = __fmul_rn(u, su);
        }
        const float h = __fmul_rn(silu_ref(g), u);  // silu(g) * u (kernels/gemm.py:197)
        const bool store = valid && (m0 + m < p.M);
        if (EPI == kEpiSiluBf16) {
          if (store)
            reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<long long>(m0 + m) * p.ldo + n] =
                __float2bfloat16_rn(h);
        } else {
          // kernels/gemm.py:198-211: round through bf16, per-64 amax, int8 codes
          const float hb = bf16_round_f32(h);
          float amax = fabsf(hb);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
          if (lane == 0) xchg[(c >> 5) * MR + m] = amax;
          named_bar_sync(2, kTileN);
          const int wp = (c >> 5) ^ 1;  // partner warp of the same 64-column group
          amax = fmaxf(amax, xchg[wp * MR + m]);
          const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
          const int8_t q = round_i8(__fdiv_rn(hb, sc));
          if (store) {
            p.out_q[static_cast<long long>(m0 + m) * p.n_q + n] = q;
            if ((c & 63) == 0) p.out_s[static_cast<long long>(m0 + m) * (p.n_q / 64) + n / 64] = sc;
          }
        }
      }
    }
  }
  cluster.sync();
}

}  // namespace qlin
