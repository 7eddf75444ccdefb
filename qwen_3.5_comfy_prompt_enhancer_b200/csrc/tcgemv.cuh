// Weight-streaming tensor-core kernel (tcgen05, kind::i8) for the quantised
// hot path at small M (decode and short prefill chunks; up to 32 activation
// rows per row block).
//
// Orientation.  The MMA computes D[n, m] = sum_k W[k, n] * a[m, k] with the
// weight tile as operand A (M_mma = 128 output columns, MN-major: the
// engine's [K, N] weight rows are N-contiguous, which tcgen05 reads directly
// through a 128-byte-swizzled MN-major descriptor -- no transpose anywhere)
// and the activations as operand B (N_mma = 16 or 32 rows, K-major, loaded by
// one TMA into the 128-byte-swizzled layout).  The int32 accumulator of each
// 64-element activation group lives in tensor memory; drain warps read it
// back, apply the per-(row, group) activation scale and accumulate fp32 in
// registers -- the reference's per-64-block `tl.dot` followed by
// `out += acc * a_s` (kernels/gemm.py:40-49, kernels/w4.py:125-130).
// Integer sums are exact; only the fp32 order of the K-split reduction
// differs from the reference.
//
// Batches.  The CTA's K range (nst groups of 64) is processed in batches of
// `bs` groups.  Every hand-off between warps -- weights landed, weights
// unpacked, accumulators ready, slots free -- is one mbarrier phase per
// batch, not per group: a completed-phase wait costs a converged warp
// ~150-200 cycles and a tcgen05.commit ~60, against ~60-90 for one
// 128x16x32 MMA, so per-group hand-offs would dominate the issue loop.  When
// the whole K range fits (the usual decode case) there is a single batch.
//
// Warp roles (one CTA = one 128-column tile x one K range); every role runs
// as a converged warp and an elected lane issues TMA / MMA / commit:
//   warp 0      TMA producer: weight rows (+ W4 group scales / zeros) of a
//               batch into a ring slot.  The first ring-full is requested
//               before the CTA-wide set-up barrier (weights never depend on
//               the preceding kernel).
//   warp 1      tensor-memory owner and MMA issuer.  After the grid
//               dependency it loads the activation tile by TMA.
//   warps 2-5   drain: activation scales, then per batch read the int32
//               accumulators (thread = output column), rescale, sum; finally
//               the epilogue.
//   warps 6-9   (W4 only) unpack: packed nibbles -> uint8 rows of swizzled A
//               tiles.  Low nibble of packed row j is K = 2j, high nibble
//               K = 2j+1.  The MMA multiplies unsigned nibbles with signed
//               activations; the zero point is removed exactly in integers
//               by the drain: sum(a*(nib - z)) = sum(a*nib) - z*sum(a).
//
// Split-K across the CTAs of a thread-block cluster: ranks 1..split-1 push
// their fp32 partial sums into rank 0's shared memory with asynchronous
// remote stores that complete rank 0's receive barrier (distributed shared
// memory, no global scratch) and exit; rank 0 adds them in rank order and
// runs the epilogue.  PDL: weights stream before griddepcontrol.wait.
#pragma once

#include <cooperative_groups.h>

#include "args.cuh"
#include "qlin_common.cuh"

namespace qlin {

constexpr int kTcWarpTma = 0;
constexpr int kTcWarpMma = 1;
constexpr int kTcWarpDrain = 2;   // 4 warps
constexpr int kTcWarpUnpack = 6;  // 4 warps (W4)
constexpr int kDrainThreads = 128;

// Tensor-memory columns one CTA may hold: two CTAs share an SM (this launch
// and the next one, under programmatic dependent launch).
constexpr uint32_t kTmemBudget = 256;

__host__ __device__ constexpr int tc_threads(int wb) { return (wb == 8 ? 6 : 10) * 32; }

struct TcLayout {
  uint32_t nsub, wtile, sztile, atile, raw_stream, raw_stage, raw_off, sz_off, a_off, b_off, nbox, as_off, asum_off,
      part_off, part_bytes, op_bytes, xchg_off, bar_off, tmem_slot_off, total, tmem_cols, per_buf;
};

__host__ __device__ inline uint32_t pow2_at_least(uint32_t x) {
  uint32_t p = 32;
  while (p < x) p <<= 1;
  return p;
}

// Shared-memory carve-up relative to a 1024-byte aligned base; `total`
// includes 1 KB of alignment slack.  bs groups per batch, rb weight-ring
// slots, ab unpacked-ring slots (W4), nbb accumulator batches.  With
// `alias`, the partial sums of ranks 1..split-1 are received in rank 0's MMA
// operand region (unpacked ring for W4, weight ring for W8) once rank 0's
// MMAs have completed, instead of a region of their own.
__host__ __device__ inline TcLayout tc_layout(int wb, int mr, int ns, int wgrp, int gmax, int bs, int rb, int ab,
                                              int nbb, int split, int alias) {
  const int nm = mr < 16 ? 16 : mr;
  TcLayout L;
  L.nsub = (wb == 4 && wgrp == 32) ? 2 : 1;
  // Per (group, stream): the weight tile as loaded (W8: 64 K rows; W4: 32
  // packed rows; each a 1024-byte aligned 128-byte-swizzled tile), the W4
  // group scales (bf16) + zeros (uint8), and the W4 operand-ring tile (the
  // unpacked K rows 0-31 of the group; rows 32-63 are unpacked in place over
  // the packed tile).
  L.wtile = wb == 8 ? 64 * kTileN : 32 * kTileN;
  L.sztile = wb == 8 ? 0 : L.nsub * kTileN * 3;
  L.atile = wb == 8 ? 0 : 32 * kTileN;
  L.raw_stream = L.wtile + L.sztile;
  L.raw_stage = ns * L.raw_stream;
  uint32_t off = 0;
  L.raw_off = off;
  off = align_up(off + rb * bs * ns * L.wtile, 1024);
  L.sz_off = off;
  off = align_up(off + rb * bs * ns * L.sztile, 1024);
  L.a_off = off;
  if (wb == 4) off = align_up(off + ab * bs * ns * L.atile, 1024);
  // Activation operand: boxes of 128 K (one swizzle row) x nm rows.
  L.b_off = off;
  L.nbox = (gmax + 1) / 2;
  off = align_up(off + L.nbox * nm * 128, 1024);
  L.as_off = off;
  off = align_up(off + gmax * nm * 4, 16);
  L.asum_off = off;
  off = align_up(off + (wb == 4 ? gmax * 2 * nm * 4 : 0), 16);
  // Partial sums pushed by the cluster's ranks 1..split-1 into rank 0.
  L.part_bytes = (split > 1 ? split - 1 : 0) * ns * mr * kTileN * 4;
  L.op_bytes = wb == 4 ? ab * bs * ns * L.atile : rb * bs * ns * L.wtile;
  if (alias) {
    L.part_off = wb == 4 ? L.a_off : L.raw_off;
  } else {
    L.part_off = off;
    off = align_up(off + L.part_bytes, 16);
  }
  L.xchg_off = off;
  off = align_up(off + 4 * mr * 4, 16);
  L.bar_off = off;
  off = align_up(off + 8 * (2 * rb + 2 * ab + 2 * nbb + 3), 16);
  L.tmem_slot_off = off;
  off += 16;
  L.total = off + 1024;
  L.per_buf = ns * L.nsub * nm;
  L.tmem_cols = pow2_at_least(nbb * bs * L.per_buf);
  return L;
}

template <int WB, int MR, int EPI>
__global__ void __launch_bounds__(tc_threads(WB), 1) tc_gemv_kernel(const __grid_constant__ GemvArgs p) {
  namespace cg = cooperative_groups;
  constexpr int NS = (EPI == kEpiOut) ? 1 : 2;
  constexpr int NM = MR < 16 ? 16 : MR;   // MMA N (activation rows, padded)
  constexpr int LDN = MR <= 8 ? 8 : MR;   // TMEM columns read per accumulator
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  if (threadIdx.x == 0) QLIN_TL(p, 0);
  const int BS = p.bs, RB = p.rb, NBB = p.nbb;
  const int AB = WB == 4 ? p.ab : 0;
  const int ab_div = AB > 0 ? AB : 1;  // W8 has no unpacked ring
  const TcLayout L = tc_layout(WB, MR, NS, p.wgrp, p.gmax, BS, RB, AB, NBB, p.split, p.part_alias);
  const int NSUB = static_cast<int>(L.nsub);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + RB;
  uint64_t* afull = empty + RB;
  uint64_t* aempty = afull + AB;
  uint64_t* tfull = aempty + AB;
  uint64_t* tempty = tfull + NBB;
  uint64_t* bfull = tempty + NBB;
  uint64_t* recv = bfull + 1;   // rank 0: partial sums of the other ranks landed
  uint64_t* ready = recv + 1;   // ranks > 0: rank 0's operand region is free (part_alias)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem_slot_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = blockIdx.x;
  const int tile = blockIdx.y;
  const int m0 = blockIdx.z * NM;

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
  const int nbatch = (nst + BS - 1) / BS;
  auto batch_len = [&](int b) { return (b + 1) * BS <= nst ? BS : nst - b * BS; };

  uint8_t* raw = smem + L.raw_off;
  uint8_t* szr = smem + L.sz_off;
  uint8_t* abuf = smem + L.a_off;
  uint8_t* bop = smem + L.b_off;
  float* ass = reinterpret_cast<float*>(smem + L.as_off);
  int* asum = reinterpret_cast<int*>(smem + L.asum_off);
  float* part = reinterpret_cast<float*>(smem + L.part_off);
  // Weight tile, W4 scales + zeros, and W4 operand-ring tile of (ring slot,
  // group-in-batch, stream).
  auto raw_w = [&](int rs, int j, int s) { return raw + ((rs * BS + j) * NS + s) * L.wtile; };
  auto raw_sz = [&](int rs, int j, int s) { return szr + ((rs * BS + j) * NS + s) * L.sztile; };
  auto a_tile = [&](int as, int j, int s) { return abuf + ((as * BS + j) * NS + s) * L.atile; };

  // Drain thread -> output column of this tile (TMEM lane 32*(warp%4) + lane).
  const bool is_drain = warp >= kTcWarpDrain && warp < kTcWarpDrain + 4;
  const int q = warp & 3;
  const int c = 32 * q + lane;
  const bool epi_thread = is_drain && rank == 0;
  const int en = n0 + c;
  const bool evalid = epi_thread && en < S0.n;
  float pre_s0 = 1.0f, pre_s1 = 1.0f;
  if (WB == 8 && evalid) {
    pre_s0 = __ldg((NS == 1 ? S0.bs : p.seg[0].bs) + en);
    if (NS == 2) pre_s1 = __ldg(p.seg[1].bs + en);
  }
  float pre_res[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) pre_res[m] = 0.0f;

  // ---------------------------------------------------------------- set-up
  uint32_t group_bytes = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const GemvSeg& sg = NS == 1 ? S0 : p.seg[s];
    group_bytes += WB == 8 ? 64 * kTileN : 32 * kTileN + L.nsub * kTileN * 2 + (sg.has_z ? L.nsub * kTileN : 0);
  }
  auto issue_batch = [&](int b, uint64_t pol) {
    const int rs = b % RB;
    const int nb = batch_len(b);
    mbar_arrive_expect_tx(full + rs, group_bytes * nb);
    for (int j = 0; j < nb; ++j) {
      const int g = g0 + b * BS + j;
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        const GemvSeg& sg = NS == 1 ? S0 : p.seg[s];
        uint8_t* dst = raw_w(rs, j, s);
        if (WB == 8) {
          tma_load_2d(dst, &sg.tw, n0, g * 64, full + rs, pol);
        } else {
          tma_load_2d(dst, &sg.tw, n0, g * 32, full + rs, pol);
          const int srow = (g * 64) / p.wgrp;
          uint8_t* sz = raw_sz(rs, j, s);
          tma_load_2d(sz, &sg.ts, n0, srow, full + rs, pol);
          if (sg.has_z) tma_load_2d(sz + L.nsub * kTileN * 2, &sg.tz, n0, srow, full + rs, pol);
        }
      }
    }
  };
  const int prefill = nbatch < RB ? nbatch : RB;

  if (warp == kTcWarpTma) {
    if (lane == 0) {
      for (int i = 0; i < RB; ++i) {
        mbar_init(full + i, 1);
        mbar_init(empty + i, WB == 8 ? 1 : 8);
      }
      for (int i = 0; i < AB; ++i) {
        mbar_init(afull + i, 128);
        mbar_init(aempty + i, 1);
      }
      for (int i = 0; i < NBB; ++i) {
        mbar_init(tfull + i, 1);
        mbar_init(tempty + i, kDrainThreads);
      }
      mbar_init(bfull, 1);
      mbar_init(recv, 1);
      mbar_init(ready, 1);
      fence_mbar_init();
      // Rank 0 expects every other rank's partial sums as asynchronous
      // remote stores that complete the receive barrier's byte count.
      if (p.split > 1 && rank == 0)
        mbar_arrive_expect_tx(recv, static_cast<uint32_t>((p.split - 1) * kDrainThreads * NS * MR * 4));
    }
    __syncwarp();
    if (elect_one()) {
      const uint64_t pol = l2_policy_evict_first();
      for (int b = 0; b < prefill; ++b) issue_batch(b, pol);
    }
    __syncwarp();
  } else if (warp == kTcWarpMma) {
    tmem_alloc(tmem_slot, L.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Let the next launch's CTAs be placed now, so that they request their
  // weights while this launch waits and computes.  No CTA of this launch can
  // then wait on a later launch: the next grid starts only once every CTA of
  // this one has passed this point, after its tensor-memory allocation.
  pdl_launch_dependents();
  // Every rank's barriers are initialised (and rank 0's receive barrier armed)
  // before any rank signals another.  Waiting here, with the weights already
  // in flight, keeps the cluster barrier off the tail of the launch.
  if (p.split > 1) {
    cluster_arrive_relaxed();
    cluster_wait();
  }
  const uint32_t tbase = *tmem_slot;
  if (threadIdx.x == 0) QLIN_TL(p, 1);

  float acc[NS][MR];  // drain threads: this CTA's partial sums for output column c
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[s][m] = 0.0f;

  // TMEM accumulator column of (batch buffer, group-in-batch, stream, sub-block).
  auto tcol = [&](int tb, int j, int s, int sub) -> uint32_t {
    return static_cast<uint32_t>((((tb * BS + j) * NS + s) * NSUB + sub) * NM);
  };

  if (warp == kTcWarpTma) {
    // ------------------------------------------------------------------ producer
    const uint64_t pol = l2_policy_evict_first();
    for (int b = prefill; b < nbatch; ++b) {
      const int rs = b % RB;
      if (!mbar_wait(empty + rs, ((b / RB) & 1) ^ 1)) {
        if (lane == 0) record_fault(p.fault, kFaultEmptyWait);
        break;
      }
      if (elect_one()) issue_batch(b, pol);
      __syncwarp();
    }
  } else if (warp == kTcWarpMma) {
    // ------------------------------------------------------------------ MMA issuer
    pdl_wait();
    if (lane == 0) QLIN_TL(p, 2);
    if (elect_one()) {
      mbar_arrive_expect_tx(bfull, L.nbox * NM * 128);
      const uint64_t pol = l2_policy_evict_last();
      for (uint32_t bx = 0; bx < L.nbox; ++bx)
        tma_load_2d(bop + bx * NM * 128, &p.ta, g0 * 64 + 128 * bx, m0, bfull, pol);
    }
    __syncwarp();
    constexpr uint32_t idesc = idesc_i8(128, NM, WB == 8, true, true, false);
    bool ok = mbar_wait(bfull, 0);
    if (lane == 0) QLIN_TL(p, 3);
    for (int b = 0; ok && b < nbatch; ++b) {
      const int rs = b % RB;
      const int as = WB == 4 ? b % ab_div : 0;
      const int tb = b % NBB;
      if (WB == 8) ok = mbar_wait(full + rs, (b / RB) & 1);
      else ok = mbar_wait(afull + as, (b / ab_div) & 1);
      if (b >= NBB) ok = ok && mbar_wait(tempty + tb, ((b / NBB) & 1) ^ 1);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        const int nb = batch_len(b);
        for (int j = 0; j < nb; ++j) {
          const int i = b * BS + j;  // group within the CTA's K range
          const uint32_t b_row = smem_u32(bop + (i >> 1) * NM * 128) + (i & 1) * 64;
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            // kk = 0 / 1: K rows 0-31 / 32-63 of the group: W8 rows of the
            // weight tile; W4 the ring tile, then the tile unpacked in place.
            const uint32_t w_addr = smem_u32(raw_w(rs, j, s));
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint32_t src = WB == 8 ? w_addr + 4096 * kk : (kk == 0 ? smem_u32(a_tile(as, j, s)) : w_addr);
              const uint64_t ad = smem_desc(src, 8192, 1024, kLayoutSw128);
              const uint64_t bd = smem_desc(b_row + 32 * kk, 16, 1024, kLayoutSw128);
              const uint32_t d = tbase + tcol(tb, j, s, NSUB == 2 ? kk : 0);
              tc_mma_i8(d, ad, bd, idesc, NSUB == 2 ? 0u : static_cast<uint32_t>(kk));
            }
          }
        }
        tc_commit(tfull + tb);
        tc_commit(WB == 8 ? empty + rs : aempty + as);
      }
      __syncwarp();
    }
    if (lane == 0) QLIN_TL(p, 4);
    if (!ok && lane == 0) record_fault(p.fault, kFaultMmaWait);
  } else if (is_drain) {
    // ------------------------------------------------------------------ drain
    const int td = threadIdx.x - kTcWarpDrain * 32;
    pdl_wait();
    if (EPI == kEpiOut && evalid && p.res) {
      const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(p.res);
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m0 + m < p.M)
          pre_res[m] = __bfloat162float(res[static_cast<long long>(m0 + m) * p.ldr + S0.out_col + en]);
    }
    for (int idx = td; idx < NM * nst; idx += kDrainThreads) {
      const int m = idx % NM, gl = idx / NM;
      ass[gl * NM + m] = (m0 + m < p.M) ? __ldg(p.a_s + static_cast<long long>(m0 + m) * G + g0 + gl) : 0.0f;
    }
    bool ok = true;
    if (WB == 4) {
      // Sum of the activation over each 32-K half group, read from the
      // swizzled B tile (rows past M are zero-filled by the TMA).
      ok = mbar_wait(bfull, 0);
      for (int idx = td; ok && idx < NM * nst * 2; idx += kDrainThreads) {
        const int m = idx % NM, gh = idx / NM;
        const int gl = gh >> 1, h = gh & 1;
        const int c0 = (gl & 1) * 4 + h * 2;  // logical 16-byte chunk in the 128-byte row
        const uint8_t* row = bop + (gl >> 1) * NM * 128 + m * 128;
        const int4 v0 = *reinterpret_cast<const int4*>(row + ((c0 ^ (m & 7)) << 4));
        const int4 v1 = *reinterpret_cast<const int4*>(row + (((c0 + 1) ^ (m & 7)) << 4));
        int sa = 0;
        sa = dp4a_ss(v0.x, 0x01010101, sa); sa = dp4a_ss(v0.y, 0x01010101, sa);
        sa = dp4a_ss(v0.z, 0x01010101, sa); sa = dp4a_ss(v0.w, 0x01010101, sa);
        sa = dp4a_ss(v1.x, 0x01010101, sa); sa = dp4a_ss(v1.y, 0x01010101, sa);
        sa = dp4a_ss(v1.z, 0x01010101, sa); sa = dp4a_ss(v1.w, 0x01010101, sa);
        asum[gh * NM + m] = sa;
      }
    }
    named_bar_sync(1, kDrainThreads);  // ass / asum visible to all drain threads

    const uint32_t lane_base = tbase + (static_cast<uint32_t>(32 * q) << 16);
    for (int b = 0; ok && b < nbatch; ++b) {
      const int rs = b % RB;
      const int tb = b % NBB;
      if (WB == 4) ok = mbar_wait(full + rs, (b / RB) & 1);
      ok = ok && mbar_wait(tfull + tb, (b / NBB) & 1);
      if (!ok) break;
      tc_fence_after();
      const int nb = batch_len(b);
      for (int j = 0; j < nb; ++j) {
        const int i = b * BS + j;
        uint32_t r[NS][2][LDN];
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          tmem_ld32<LDN>(lane_base + tcol(tb, j, s, 0), r[s][0]);
          if (WB == 4 && NSUB == 2) tmem_ld32<LDN>(lane_base + tcol(tb, j, s, 1), r[s][1]);
        }
        tc_wait_ld();
        const float* as_g = ass + i * NM;
        if (WB == 8) {
          // out += float(int32 group sum) * a_s[m, kb]   (kernels/gemm.py:43-45)
#pragma unroll
          for (int s = 0; s < NS; ++s)
#pragma unroll
            for (int m = 0; m < MR; ++m)
              acc[s][m] = __fadd_rn(acc[s][m], __fmul_rn(__int2float_rn(static_cast<int>(r[s][0][m])), as_g[m]));
        } else {
          // out += float(int32 sub-block sum) * (a_s * ws)   (kernels/w4.py:103-104)
          const int* asum_g = asum + i * 2 * NM;
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            const GemvSeg& sg = NS == 1 ? S0 : p.seg[s];
            const uint8_t* st = raw_sz(rs, j, s);
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(st);
            const uint8_t* zz = st + L.nsub * kTileN * 2;
            for (int sub = 0; sub < NSUB; ++sub) {
              const float ws = bf16_bits_to_f32(sc[sub * kTileN + c]);
              const int z = sg.has_z ? static_cast<int>(zz[sub * kTileN + c]) : 8;
#pragma unroll
              for (int m = 0; m < MR; ++m) {
                const int sa = NSUB == 2 ? asum_g[sub * NM + m] : asum_g[m] + asum_g[NM + m];
                const int v = static_cast<int>(r[s][sub][m]) - z * sa;
                const float t = __fmul_rn(as_g[m], ws);
                acc[s][m] = __fadd_rn(acc[s][m], __fmul_rn(__int2float_rn(v), t));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty + tb);
      if (WB == 4) {
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + rs);
      }
    }
    if (td == 0) QLIN_TL(p, 5);
    if (!ok && lane == 0) record_fault(p.fault, kFaultFullWait);
    if (p.part_alias && rank == 0) {
      // The last accumulator batch was observed: every MMA of this CTA has
      // completed, so its operand region is free to receive the other
      // ranks' partial sums.
      if (ok && td == 0)
        for (int r = 1; r < p.split; ++r) mbar_arrive_remote(map_to_rank(smem_u32(ready), r));
    }
  } else if constexpr (WB == 4) {
    // ------------------------------------------------------------------ W4 unpack
    // Packed row r of a group's tile holds k = 2r (low nibbles) and 2r + 1
    // (high nibbles) for 128 columns.  K rows 0-31 (packed rows 0-15) go to
    // the ring tile and K rows 32-63 (packed rows 16-31) are written in place
    // over the packed tile, both in the 128-byte-swizzled MN-major operand
    // layout the tensor-map load produced.  Thread u owns packed rows u/8 and
    // u/8 + 16 in 16-column chunk u%8; the in-place writes wait on a barrier
    // of the 128 unpack threads until every packed row has been read.
    const int u = threadIdx.x - kTcWarpUnpack * 32;
    const int pr = u >> 3, ch = u & 7;
    auto chunk = [&](int r) { return r * kTileN + ((ch ^ (r & 7)) << 4); };
    auto lo4 = [](const uint4& v) {
      return make_uint4(v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu);
    };
    auto hi4 = [](const uint4& v) {
      return make_uint4((v.x >> 4) & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                        (v.w >> 4) & 0x0F0F0F0Fu);
    };
    constexpr int kChunkTiles = 4;  // tiles read per barrier
    for (int b = 0; b < nbatch; ++b) {
      const int rs = b % RB;
      const int as = b % AB;
      const bool waited = mbar_wait(full + rs, (b / RB) & 1) && mbar_wait(aempty + as, ((b / AB) & 1) ^ 1);
      const int nt = batch_len(b) * NS;
      bool ok = true;
      for (int t0 = 0; t0 < nt; t0 += kChunkTiles) {
        uint4 v0[kChunkTiles], v1[kChunkTiles];
#pragma unroll
        for (int q = 0; q < kChunkTiles; ++q) {
          if (t0 + q >= nt) break;
          const uint8_t* wt = raw_w(rs, (t0 + q) / NS, (t0 + q) % NS);
          v0[q] = *reinterpret_cast<const uint4*>(wt + chunk(pr));
          v1[q] = *reinterpret_cast<const uint4*>(wt + chunk(pr + 16));
        }
        // (the first barrier of a batch also agrees on the waits' outcome, so
        // that all 128 threads leave together after a timed-out wait)
        if (t0 == 0) ok = named_bar_and(3, 128, waited);
        else named_bar_sync(3, 128);
        if (!ok) break;
#pragma unroll
        for (int q = 0; q < kChunkTiles; ++q) {
          if (t0 + q >= nt) break;
          const int j = (t0 + q) / NS, s = (t0 + q) % NS;
          uint8_t* wt = raw_w(rs, j, s);
          uint8_t* at = a_tile(as, j, s);
          *reinterpret_cast<uint4*>(at + chunk(2 * pr)) = lo4(v0[q]);
          *reinterpret_cast<uint4*>(at + chunk(2 * pr + 1)) = hi4(v0[q]);
          *reinterpret_cast<uint4*>(wt + chunk(2 * pr)) = lo4(v1[q]);
          *reinterpret_cast<uint4*>(wt + chunk(2 * pr + 1)) = hi4(v1[q]);
        }
      }
      if (!ok) {
        if (lane == 0) record_fault(p.fault, kFaultFullWait);
        break;
      }
      fence_proxy_async_smem();
      mbar_arrive(afull + as);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + rs);
    }
  }

  // ------------------------------------------------------------------ cluster combine + epilogue
  __syncwarp();
  tc_fence_before();
  __syncthreads();  // every tensor-memory read has completed
  tc_fence_after();
  if (warp == kTcWarpMma) tmem_dealloc(tbase, L.tmem_cols);
  // Ranks 1..split-1 push their partial sums into rank 0's shared memory with
  // asynchronous stores, each completing 4 bytes of rank 0's receive barrier
  // (armed at set-up with the total), then exit: nothing reads their shared
  // memory, so no closing cluster barrier.  This relies on rank 0 outliving
  // every remote store: it exits only after its receive barrier completed (or
  // after two bounded waits for it, on the fault path).
  if (is_drain && rank > 0) {
    bool go = true;
    if (p.part_alias && !mbar_wait_cluster(ready, 0)) {
      go = false;
      if (lane == 0) record_fault(p.fault, kFaultFullWait);
    }
    if (go) {
      const uint32_t slot0 = smem_u32(part + static_cast<size_t>(rank - 1) * NS * MR * kTileN);
      const uint32_t dst = map_to_rank(slot0, 0);
      const uint32_t rbar = map_to_rank(smem_u32(recv), 0);
#pragma unroll
      for (int s = 0; s < NS; ++s)
#pragma unroll
        for (int m = 0; m < MR; ++m) st_async_f32(dst + ((s * MR + m) * kTileN + c) * 4, acc[s][m], rbar);
    }
    if (c == 0) QLIN_TL(p, 6);
  }
  if (epi_thread) {
    const int n = en;
    const bool valid = n < S0.n;
    // Fixed summation order: rank 0, then ranks 1, 2, ...
    float vs[NS][MR];
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m) vs[s][m] = acc[s][m];
    if (p.split > 1 && !mbar_wait_cluster(recv, 0)) {
      if (lane == 0) record_fault(p.fault, kFaultFullWait);
      // The other ranks exit without a closing cluster barrier, so this CTA
      // must outlive their remote stores into its shared memory.  After a
      // timed-out receive it waits once more (bounded) for late partial sums
      // before it exits; the launch's result is wrong either way and the
      // fault word says so.
      mbar_wait_cluster(recv, 0);
    } else {
      for (int r = 1; r < p.split; ++r) {
        const float* rp = part + static_cast<size_t>(r - 1) * NS * MR * kTileN;
#pragma unroll
        for (int s = 0; s < NS; ++s)
#pragma unroll
          for (int m = 0; m < MR; ++m) vs[s][m] = __fadd_rn(vs[s][m], rp[(s * MR + m) * kTileN + c]);
      }
    }
    if (c == 0) QLIN_TL(p, 6);
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
      float* xchg = reinterpret_cast<float*>(smem + L.xchg_off);
      float hb[MR], amax[MR];
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float g = vs[0][m], uu = vs[1][m];
        if (WB == 8) {
          g = __fmul_rn(g, pre_s0);
          uu = __fmul_rn(uu, pre_s1);
        }
        const float h = __fmul_rn(silu_ref(g), uu);  // silu(g) * u (kernels/gemm.py:197)
        if (EPI == kEpiSiluBf16) {
          if (valid && (m0 + m < p.M))
            reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<long long>(m0 + m) * p.ldo + n] =
                __float2bfloat16_rn(h);
        } else {
          // kernels/gemm.py:198-211: round through bf16, per-64 amax, int8 codes
          hb[m] = bf16_round_f32(h);
          amax[m] = fabsf(hb[m]);
        }
      }
      if (EPI == kEpiSiluQuant) {
        // every row's warp amax, one exchange with the other warp of each
        // 64-column group for all rows, then the codes
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int m = 0; m < MR; ++m) amax[m] = fmaxf(amax[m], __shfl_xor_sync(0xffffffffu, amax[m], o));
        if (lane == 0)
#pragma unroll
          for (int m = 0; m < MR; ++m) xchg[q * MR + m] = amax[m];
        named_bar_sync(2, kDrainThreads);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const float am = fmaxf(amax[m], xchg[(q ^ 1) * MR + m]);  // the other warp of this 64-column group
          const float sc = fmaxf(__fdiv_rn(am, 127.0f), 1e-8f);
          const int8_t qv = round_i8(__fdiv_rn(hb[m], sc));
          if (valid && (m0 + m < p.M)) {
            p.out_q[static_cast<long long>(m0 + m) * p.n_q + n] = qv;
            if ((c & 63) == 0) p.out_s[static_cast<long long>(m0 + m) * (p.n_q / 64) + n / 64] = sc;
          }
        }
      }
    }
    if (c == 0) QLIN_TL(p, 7);
  }
}

}  // namespace qlin
