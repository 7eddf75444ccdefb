// Weight-streaming GEMV on CUDA cores for decode rows (M <= 2): the small-M
// entry points (gemm_i8 / gemm_w4 + residual, proj3(_w4), the fused gate/up
// epilogues).
//
// Why not the tensor cores here.  At M <= 2 the work per weight byte is tiny
// and what counts is the time from the grid dependency to the last store.
// This kernel keeps W4 nibbles packed (4 KB per 64-K group and 128 columns,
// half of what an unpacked MMA operand needs) and decodes them in registers;
// there is no operand hand-off chain.
//
// Two weight modes:
//  * resident -- every weight of the CTA's K range is requested before the
//    dependency, so under programmatic dependent launch the whole stream
//    overlaps the preceding kernel;
//  * ring -- each warp owns `ring` slots; the first `ring` items of every warp
//    are requested before the dependency and a slot is refilled as soon as
//    its warp has used it (long launches: tens of MB of weights).
//
// Work split.  CTA = one 128-column tile x one K part; a tile's K is cut into
// split x kout parts: `split` CTAs of a thread-block cluster combine their
// partial sums through distributed shared memory, and the `kout` clusters of
// a tile through a device workspace (the last cluster to arrive adds them and
// runs the epilogue).  Lane l of every warp owns columns 4l .. 4l+3; warp w
// owns the (group, stream) items w, w + 8, ... of the CTA's K part.  Per item
// the int32 dot of each (row, column) over the group's 64 K (W4 groups of 32:
// per 32-K half) is complete inside one thread before the fp32 epilogue of
// the reference:
//   W8: acc += float(I) * a_s[m, kb]                   (kernels/gemm.py:43-45)
//   W4: acc += float(I - z * sum(a)) * (a_s[m, kb] * ws)  (kernels/w4.py:103-104)
// Four weight rows (4 columns each) are transposed with byte permutes so
// that dp4a reduces along K; a W4 word of 4 packed rows holds 8 K values of
// one column: the low nibbles (even K) and high nibbles (odd K) meet
// activation words pre-split by K parity (dp4a.u32.s32, unsigned nibbles).
// The zero point is removed exactly: sum(a (nib - z)) = sum(a nib) - z sum(a).
//
// Reduction order (fixed): per warp its items in order, then the 8 warps in
// order, then the cluster's ranks in order, then the clusters in K order;
// only this fp32 order differs from the reference's ascending-K sum.
#pragma once

#include "args.cuh"
#include "qlin_common.cuh"

namespace qlin {

constexpr int kRgThreads = 256;
constexpr int kRgWarps = kRgThreads / 32;
// Blocks of a weight item unrolled together in the dot loop (W8: 16 blocks of
// 4 K rows, W4: 4 blocks of 8 K per 32-K half).  Measured on B200 (graph
// replay, us, full unroll vs 4 / 2): config-2 W4 gate/up 4.6 vs 5.6, down 3.8
// vs 4.6, qkv 3.0 vs 3.7, config-1 W8 3.3 vs 3.5 at M = 1; W4 gate/up 8.2 vs
// 9.0 at M = 4.
#ifndef QLIN_DP_UNROLL_W8
#define QLIN_DP_UNROLL_W8 16
#endif
#ifndef QLIN_DP_UNROLL_W4
#define QLIN_DP_UNROLL_W4 4
#endif
constexpr int kDpUnrollW8 = QLIN_DP_UNROLL_W8;
constexpr int kDpUnrollW4 = QLIN_DP_UNROLL_W4;

// Device workspace of the cross-cluster K parts: per slot, fp32 partial sums
// [tile][kout][stream][row][128] and one arrival counter per tile.  The host
// rotates launches over the slots; a counter is reset by the launch's last
// arrival, so a slot is free again once its launch has completed.
constexpr int kDpWsSlots = 4;
constexpr int kDpWsFloats = 1 << 17;
constexpr int kDpWsTiles = 1024;
static __device__ __align__(256) float g_dp_ws[kDpWsSlots][kDpWsFloats];
static __device__ __align__(256) unsigned g_dp_cnt[kDpWsSlots][kDpWsTiles];

// Column-split layer only (kEpiOut, one segment): the activation rows come
// from the ranks' flagged words of h in this rank's exchange buffer instead of
// a_q / a_s, and every output row also goes to every rank's exchange buffer of
// the output as flagged words (the layouts of qlin_peer_allgather_ll: codes
// [M][kloc] then scales [M][kloc / 64] per sender; outputs [M][N] bf16).
constexpr int kDpPeerMax = 8;
struct DpPeer {
  const uint8_t* rx;          // this rank's exchange buffer of h, or null
  long long rx_slot;          // bytes of one sender slot
  long long rx_off_s;         // byte offset of the scale words in a slot (codes at 0)
  const unsigned* rx_state;   // call number = rx_state[0] + 1
  int rx_kloc;                // h columns each rank sends (multiple of 128)
  int8_t* rx_hq;              // optional copy of the received rows [M][K] (tile 0 writes it), or null
  float* rx_hs;               // and of their scales [M][K / 64]
  uint8_t* tx[kDpPeerMax];    // every rank's exchange buffer of the output, or null
  long long tx_slot;
  const unsigned* tx_state;   // call number = tx_state[0] + 1
  int world, rank;
};

struct DpArgs {
  CUtensorMap tw[3];   // weights, plain (unswizzled) boxes: W8 128 columns x 64 rows; W4 128 x 32 packed rows
  CUtensorMap ts[3];   // W4 group scales (bf16), box 128 x nsub
  CUtensorMap tz[3];   // W4 zeros (uint8), box 128 x nsub
  GemvSeg seg[3];      // n, out_col, tile_begin, has_z, bs (W8)
  int nseg;
  const int8_t* a_q;   // [M, K]
  const float* a_s;    // [M, K/64]
  int M, K, wgrp, split, gmax;
  int ring;            // weight slots per warp; 0: every item resident
  int kout;            // clusters per tile (K parts across clusters)
  int ws_slot;         // workspace slot (kout > 1)
  int tl_slot;         // tuning builds: phase-timeline slot of this launch (-1: none)
  void* out;
  long long ldo;
  const void* res;
  long long ldr;
  int8_t* out_q;
  float* out_s;
  int n_q;
  DpPeer peer;
  unsigned* fault;
};

// Shared-memory carve-up (host and device): the weight slots (every (group,
// stream) item, or `ring` per warp), the K-part activation rows, the
// cross-warp reduction (over the weights once they are used), the partial
// sums received from the other ranks, barriers.
struct DpLayout {
  uint32_t item, wbytes, sbytes, act_off, as_off, part_off, xchg_off, bar_off, total;
};
__host__ __device__ inline DpLayout dp_layout(int wb, int mr, int ns, int wgrp, int gmax, int split, int ring) {
  DpLayout L;
  const int nsub = (wb == 4 && wgrp == 32) ? 2 : 1;
  L.wbytes = wb == 8 ? 64 * kTileN : 32 * kTileN;
  L.sbytes = wb == 8 ? 0 : nsub * kTileN * 3;
  L.item = align_up(L.wbytes + L.sbytes, 128);
  uint32_t off = (ring > 0 ? kRgWarps * ring : gmax * ns) * L.item;
  const uint32_t red = kRgWarps * mr * kTileN * 4;  // aliases the weights
  if (off < red) off = red;
  off = align_up(off, 128);
  L.act_off = off;
  off = align_up(off + gmax * mr * 64, 16);
  L.as_off = off;  // the K part's activation scales [m][gmax], then (W4, 16-byte aligned) sums [m][gmax][2]
  off = align_up(off + gmax * mr * 4, 16) + (wb == 4 ? align_up(gmax * mr * 8, 16) : 0);
  L.part_off = off;
  off = align_up(off + (split > 1 ? split - 1 : 0) * ns * mr * kTileN * 4, 16);
  L.xchg_off = off;
  off = align_up(off + 4 * mr * 4 + 16, 16);  // (+ the last-arrival flag)
  L.bar_off = off;
  off += 8 * (kRgWarps * (ring > 0 ? ring : 1) + 2);
  L.total = off + 128;  // alignment slack
  return L;
}

// d = c + sum_i a.u8[i] * b.s8[i]
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 4x4 byte transpose: r_i holds bytes (c0..c3) of row i; c_j returns column
// j's bytes in row order.
__device__ __forceinline__ void tr4x4(uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3, uint32_t (&c)[4]) {
  const uint32_t t0 = __byte_perm(r0, r1, 0x5140);  // a0 b0 a1 b1
  const uint32_t t1 = __byte_perm(r0, r1, 0x7362);  // a2 b2 a3 b3
  const uint32_t t2 = __byte_perm(r2, r3, 0x5140);
  const uint32_t t3 = __byte_perm(r2, r3, 0x7362);
  c[0] = __byte_perm(t0, t2, 0x5410);
  c[1] = __byte_perm(t0, t2, 0x7632);
  c[2] = __byte_perm(t1, t3, 0x5410);
  c[3] = __byte_perm(t1, t3, 0x7632);
}

template <int WB, int MR, int EPI>
__global__ void __launch_bounds__(kRgThreads, 2) dp_gemv_kernel(const __grid_constant__ DpArgs p) {
  constexpr int NS = (EPI == kEpiOut) ? 1 : 2;
  extern __shared__ __align__(128) uint8_t dp_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dp_smem_raw) + 127) & ~uintptr_t(127));
  const DpLayout L = dp_layout(WB, MR, NS, p.wgrp, p.gmax, p.split, p.ring);
  const int R = p.ring;
  const int nsub = (WB == 4 && p.wgrp == 32) ? 2 : 1;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);  // per warp (ring: per warp and slot)
  uint64_t* recv = full + kRgWarps * (R > 0 ? R : 1);
  uint64_t* abar = recv + 1;                                       // activation rows landed
  int8_t* act = reinterpret_cast<int8_t*>(smem + L.act_off);      // [m][gmax][64]: the K part of row m
  float* as_sm = reinterpret_cast<float*>(smem + L.as_off);        // [m][gmax]: its scales a_s[m, g0 + gl]
  int* asum_sm = reinterpret_cast<int*>(smem + L.as_off + align_up(MR * p.gmax * 4, 16));  // W4: [m][gmax][2]
  float* part = reinterpret_cast<float*>(smem + L.part_off);       // [rank-1][s][m][128]
  float* red = reinterpret_cast<float*>(smem);                     // [warp][m][128], over the weights

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = blockIdx.x, tile = blockIdx.y;
  int si = 0;
  if (EPI == kEpiOut) {
    if (p.nseg > 1 && tile >= p.seg[1].tile_begin) si = 1;
    if (p.nseg > 2 && tile >= p.seg[2].tile_begin) si = 2;
  }
  const GemvSeg& S0 = p.seg[si];
  const int n0 = (tile - S0.tile_begin) * kTileN;
  const int G = p.K / kGroup;
  const int nparts = p.split * p.kout;
  const int kpart = blockIdx.z * p.split + rank;
  const int g0 = static_cast<int>(static_cast<long long>(kpart) * G / nparts);
  const int g1 = static_cast<int>(static_cast<long long>(kpart + 1) * G / nparts);
  const int nst = g1 - g0;
  const int items = nst * NS;
  // weight slot of item `it` (ring: item li of warp w sits in slot li % R)
  auto item_w = [&](int it) {
    return smem + (R > 0 ? (it % kRgWarps) * R + (it / kRgWarps) % R : it) * L.item;
  };
  auto item_bytes = [&](int it) {
    const int s = NS == 1 ? si : it % NS;
    return static_cast<uint32_t>(L.wbytes +
                                 (WB == 4 ? nsub * kTileN * 2 + (p.seg[s].has_z ? nsub * kTileN : 0) : 0));
  };
  auto issue_item = [&](int it, uint64_t* bar, uint64_t pol) {
    const int gl = it / NS, s = NS == 1 ? si : it % NS;
    const int g = g0 + gl;
    uint8_t* dst = item_w(it);
    if (WB == 8) {
      tma_load_2d(dst, &p.tw[s], n0, g * 64, bar, pol);
    } else {
      tma_load_2d(dst, &p.tw[s], n0, g * 32, bar, pol);
      const int srow = (g * 64) / p.wgrp;
      tma_load_2d(dst + L.wbytes, &p.ts[s], n0, srow, bar, pol);
      if (p.seg[s].has_z) tma_load_2d(dst + L.wbytes + nsub * kTileN * 2, &p.tz[s], n0, srow, bar, pol);
    }
  };

  // ---------------------------------------------------------------- set-up: every weight requested now
  if (threadIdx.x == 0) {
    for (int w = 0; w < kRgWarps * (R > 0 ? R : 1); ++w) mbar_init(full + w, 1);
    mbar_init(recv, 1);
    mbar_init(abar, 1);
    fence_mbar_init();
    if (p.split > 1 && rank == 0)
      mbar_arrive_expect_tx(recv, static_cast<uint32_t>((p.split - 1) * kTileN * NS * MR * 4));
  }
  __syncthreads();
  if (threadIdx.x == 0) QLIN_TL(p, 0);
  const uint64_t pol = l2_policy_evict_first();
  if (lane == 0) {
    if (R == 0) {
      // warp w requests all its items, completing on its own barrier
      uint32_t bytes = 0;
      for (int it = warp; it < items; it += kRgWarps) bytes += item_bytes(it);
      if (bytes) mbar_arrive_expect_tx(full + warp, bytes);
      for (int it = warp; it < items; it += kRgWarps) issue_item(it, full + warp, pol);
    } else {
      // its first R items, one per slot
      for (int li = 0, it = warp; li < R && it < items; ++li, it += kRgWarps) {
        mbar_arrive_expect_tx(full + warp * R + li, item_bytes(it));
        issue_item(it, full + warp * R + li, pol);
      }
    }
  }
  if (threadIdx.x == 0) QLIN_TL(p, 1);
  pdl_launch_dependents();
  if (p.split > 1) {
    cluster_arrive_relaxed();
    cluster_wait();
  }

  // epilogue operands that do not depend on the previous kernel
  const int c = threadIdx.x;  // epilogue: threads 0..127 own one column each
  const bool epi_thread = threadIdx.x < kTileN && rank == 0;
  const int en = n0 + c;
  const bool evalid = epi_thread && en < S0.n;
  float pre_s0 = 1.0f, pre_s1 = 1.0f;
  if (WB == 8 && evalid) {
    pre_s0 = __ldg((NS == 1 ? S0.bs : p.seg[0].bs) + en);
    if (NS == 2) pre_s1 = __ldg(p.seg[1].bs + en);
  }

  // ---------------------------------------------------------------- activations (after the dependency)
  pdl_wait();
  if (threadIdx.x == 0) QLIN_TL(p, 2);
  float pre_res[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) pre_res[m] = 0.0f;
  if (EPI == kEpiOut && evalid && p.res) {
    const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(p.res);
#pragma unroll
    for (int m = 0; m < MR; ++m)
      if (m < p.M) pre_res[m] = __bfloat162float(res[static_cast<long long>(m) * p.ldr + S0.out_col + en]);
  }
  // the K part of every activation row, one bulk copy per row (K % 64 == 0
  // and a 16-byte aligned a_q make every row slice 16-byte aligned); rows
  // past M are never stored, so their slots are left as they are
  const int mv = p.M < MR ? p.M : MR;
  if (p.peer.rx) {
    // Column-split layer: poll the flagged words of the K part's h codes (8
    // bytes per word pair) and scales (two groups per word pair) from their
    // sender's slot until they carry this call's number (bounded).
    const DpPeer& pr = p.peer;
    const unsigned seq = pr.rx_state[0] + 1u;
    const uint8_t* base = pr.rx + static_cast<long long>(seq & 1u) * pr.world * pr.rx_slot;
    const int ncodes = mv * nst * 8, nall = ncodes + mv * nst;
    const bool keep = pr.rx_hq != nullptr && tile == 0;
    bool dead = false;
    const unsigned long long t0 = global_ns();
    for (int i = threadIdx.x; i < nall && !dead; i += kRgThreads) {
      const bool code = i < ncodes;
      int m, gl, c8 = 0;
      if (code) {
        m = i / (nst * 8);
        const int r = i - m * nst * 8;
        gl = r >> 3;
        c8 = r & 7;
      } else {
        m = (i - ncodes) / nst;
        gl = i - ncodes - m * nst;
      }
      const int k = (g0 + gl) * 64 + c8 * 8;
      const int q = k / pr.rx_kloc, kl = k - q * pr.rx_kloc;
      const uint8_t* w = base + q * pr.rx_slot +
                         (code ? (static_cast<long long>(m) * (pr.rx_kloc / 8) + kl / 8) * 16
                               : pr.rx_off_s + (static_cast<long long>(m) * (pr.rx_kloc / 128) + kl / 128) * 16);
      unsigned long long w0, w1;
      unsigned spin = 0;
      for (;;) {
        ld_sys_v2(w, w0, w1);
        if (ll_fresh(w0, seq) && ll_fresh(w1, seq)) break;
        if ((++spin & 63u) == 0 && global_ns() - t0 > wait_limit_ns()) {
          dead = true;
          break;
        }
      }
      if (dead) break;
      if (code) {
        const uint2 v = make_uint2(static_cast<unsigned>(w0), static_cast<unsigned>(w1));
        *reinterpret_cast<uint2*>(act + (m * p.gmax + gl) * 64 + c8 * 8) = v;
        if (keep) *reinterpret_cast<uint2*>(pr.rx_hq + static_cast<long long>(m) * p.K + k) = v;
      } else {
        const float sv = __uint_as_float(static_cast<unsigned>(((kl / 64) & 1) ? w1 : w0));
        as_sm[m * p.gmax + gl] = sv;
        if (keep) pr.rx_hs[static_cast<long long>(m) * G + k / 64] = sv;
      }
    }
    if (dead) record_fault(p.fault, kFaultFullWait);
    for (int i = threadIdx.x; i < (MR - mv) * nst; i += kRgThreads) as_sm[(mv + i / nst) * p.gmax + i % nst] = 0.0f;
    if (threadIdx.x == 0) mbar_arrive(abar);  // phase 0 done: the K-part combine uses phase 1
    __syncthreads();  // the received rows
  } else {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(abar, static_cast<uint32_t>(mv * nst * 64));
      for (int m = 0; m < mv; ++m)
        bulk_load(act + m * p.gmax * 64, p.a_q + static_cast<long long>(m) * p.K + g0 * 64,
                  static_cast<uint32_t>(nst * 64), abar);
    }
    // the scales of the K part, while the rows are in flight (one round trip
    // for all of them instead of one per item); rows past M scale by zero
    for (int i = threadIdx.x; i < MR * nst; i += kRgThreads) {
      const int m = i / nst, gl = i - m * nst;
      as_sm[m * p.gmax + gl] = m < p.M ? __ldg(p.a_s + static_cast<long long>(m) * G + g0 + gl) : 0.0f;
    }
    if (!mbar_wait(abar, 0)) {
      if ((threadIdx.x & 31) == 0) record_fault(p.fault, kFaultFullWait);
      mbar_wait(abar, 0);  // the copy lands before the CTA may exit
    }
  }
  if (WB == 4) {
    // Once per CTA instead of once per item and stream: every 8-byte block of
    // every row is split into its even-K and odd-K bytes (the order of the
    // low and high nibbles of a packed weight word), and each 32-K half is
    // summed for the zero points.  Rows past M hold stale bytes; they are
    // scaled by zero.
    for (int i = threadIdx.x; i < MR * nst * 2; i += kRgThreads) {
      const int m = i / (nst * 2), r = i - m * nst * 2, gl = r >> 1, h = r & 1;
      uint2* blk = reinterpret_cast<uint2*>(act + (m * p.gmax + gl) * 64 + h * 32);
      int sum = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint2 raw = blk[b];
        sum = __dp4a(static_cast<int>(raw.x), 0x01010101, __dp4a(static_cast<int>(raw.y), 0x01010101, sum));
        blk[b] = make_uint2(__byte_perm(raw.x, raw.y, 0x6420), __byte_perm(raw.x, raw.y, 0x7531));
      }
      asum_sm[(m * p.gmax + gl) * 2 + h] = sum;
    }
  }
  __syncthreads();  // as_sm (and the split rows)
  if (threadIdx.x == 0) QLIN_TL(p, 3);

  // ---------------------------------------------------------------- the dots
  // Warp w's items w, w + 8, ... all belong to stream w % NS (8 warps, NS <= 2).
  const int sw = NS == 1 ? 0 : warp % NS;
  float acc[4][MR];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[j][m] = 0.0f;
  auto dot_item = [&](int it) {
    const int gl = it / NS;
    const uint8_t* wt = item_w(it);
    float as_g[MR];  // a_s[m, group]
#pragma unroll
    for (int m = 0; m < MR; ++m) as_g[m] = as_sm[m * p.gmax + gl];
    if (WB == 8) {
      int isum[4][MR];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int m = 0; m < MR; ++m) isum[j][m] = 0;
#pragma unroll kDpUnrollW8
      for (int b = 0; b < 16; ++b) {  // 4 K rows per block
        const uint32_t* rows = reinterpret_cast<const uint32_t*>(wt + b * 4 * kTileN) + lane;
        uint32_t col[4];
        tr4x4(rows[0], rows[kTileN / 4], rows[2 * kTileN / 4], rows[3 * kTileN / 4], col);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const int aw = *reinterpret_cast<const int*>(act + (m * p.gmax + gl) * 64 + b * 4);
#pragma unroll
          for (int j = 0; j < 4; ++j) isum[j][m] = __dp4a(static_cast<int>(col[j]), aw, isum[j][m]);
        }
      }
      // out += float(int32 group sum) * a_s[m, kb]   (kernels/gemm.py:43-45)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int m = 0; m < MR; ++m)
          acc[j][m] = __fadd_rn(acc[j][m], __fmul_rn(__int2float_rn(isum[j][m]), as_g[m]));
    } else {
      const GemvSeg& sg = p.seg[NS == 1 ? si : sw];
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(wt + L.wbytes);
      const uint8_t* zz = wt + L.wbytes + nsub * kTileN * 2;
      int isum[2][4][MR];  // per 32-K half
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m = 0; m < MR; ++m) {
#pragma unroll
          for (int j = 0; j < 4; ++j) isum[h][j][m] = 0;
        }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll kDpUnrollW4
        for (int bb = 0; bb < 4; ++bb) {  // 4 packed rows = 8 K per block
          const int b = h * 4 + bb;
          const uint32_t* rows = reinterpret_cast<const uint32_t*>(wt + b * 4 * kTileN) + lane;
          uint32_t col[4];
          tr4x4(rows[0], rows[kTileN / 4], rows[2 * kTileN / 4], rows[3 * kTileN / 4], col);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            // 8 K of row m, already split by parity: (the 4 even K, the 4 odd K)
            const uint2 aw = *reinterpret_cast<const uint2*>(act + (m * p.gmax + gl) * 64 + b * 8);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              isum[h][j][m] = dp4a_us(col[j] & 0x0F0F0F0Fu, static_cast<int>(aw.x), isum[h][j][m]);
              isum[h][j][m] = dp4a_us((col[j] >> 4) & 0x0F0F0F0Fu, static_cast<int>(aw.y), isum[h][j][m]);
            }
          }
        }
      }
      int asum[2][MR];  // sum of the activations per 32-K half (zero points)
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const int2 a2 = *reinterpret_cast<const int2*>(asum_sm + (m * p.gmax + gl) * 2);
        asum[0][m] = a2.x;
        asum[1][m] = a2.y;
      }
      // out += float(int32 sub-block sum) * (a_s * ws)   (kernels/w4.py:103-104)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col_n = lane * 4 + j;
        if (nsub == 2) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float ws = bf16_bits_to_f32(sc[h * kTileN + col_n]);
            const int z = sg.has_z ? static_cast<int>(zz[h * kTileN + col_n]) : 8;
#pragma unroll
            for (int m = 0; m < MR; ++m) {
              const int v = isum[h][j][m] - z * asum[h][m];
              acc[j][m] = __fadd_rn(acc[j][m], __fmul_rn(__int2float_rn(v), __fmul_rn(as_g[m], ws)));
            }
          }
        } else {
          const float ws = bf16_bits_to_f32(sc[col_n]);
          const int z = sg.has_z ? static_cast<int>(zz[col_n]) : 8;
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const int v = isum[0][j][m] + isum[1][j][m] - z * (asum[0][m] + asum[1][m]);
            acc[j][m] = __fadd_rn(acc[j][m], __fmul_rn(__int2float_rn(v), __fmul_rn(as_g[m], ws)));
          }
        }
      }
    }
  };
  if (R == 0) {
    bool ok = true;
    if (warp < items) ok = mbar_wait(full + warp, 0);
    if (!ok) {
      if (lane == 0) record_fault(p.fault, kFaultFullWait);
      mbar_wait(full + warp, 0);  // copies still in flight land before the region is reused or the CTA exits
    }
    for (int it = warp; ok && it < items; it += kRgWarps) dot_item(it);
  } else {
    const int nw = items > warp ? (items - warp + kRgWarps - 1) / kRgWarps : 0;  // this warp's items
    for (int li = 0; li < nw; ++li) {
      const int it = warp + li * kRgWarps;
      uint64_t* bar = full + warp * R + li % R;
      if (!mbar_wait(bar, (li / R) & 1)) {
        if (lane == 0) record_fault(p.fault, kFaultFullWait);
        // copies still in flight (items li .. li + R - 1) land before the
        // region is reused or the CTA exits
        for (int k = li; k < nw && k < li + R; ++k) mbar_wait(full + warp * R + k % R, (k / R) & 1);
        break;
      }
      dot_item(it);
      __syncwarp();  // every lane's reads of the slot are done
      const int nx = li + R;
      if (lane == 0 && nx < nw) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, item_bytes(warp + nx * kRgWarps));
        issue_item(warp + nx * kRgWarps, bar, pol);
      }
    }
  }

  // ---------------------------------------------------------------- reduce: warps, then the cluster
  if (threadIdx.x == 0) QLIN_TL(p, 4);
  __syncthreads();  // every weight read -> the reduction may overwrite them
#pragma unroll
  for (int m = 0; m < MR; ++m)
    *reinterpret_cast<float4*>(red + (warp * MR + m) * kTileN + lane * 4) =
        make_float4(acc[0][m], acc[1][m], acc[2][m], acc[3][m]);
  __syncthreads();
  if (threadIdx.x >= kTileN) return;  // threads 0..127 hold one column each from here
  float vs[NS][MR];
#pragma unroll
  for (int s = 0; s < NS; ++s)
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float v = 0.0f;
#pragma unroll
      for (int w = s; w < kRgWarps; w += NS) v = __fadd_rn(v, red[(w * MR + m) * kTileN + c]);
      vs[s][m] = v;
    }
  if (threadIdx.x == 0) QLIN_TL(p, 5);
  if (rank > 0) {
    // push to rank 0, completing its receive barrier; rank 0 outlives the
    // stores (it exits only after its receive barrier completed, or after
    // two bounded waits for it on the fault path)
    const uint32_t slot0 = smem_u32(part + static_cast<size_t>(rank - 1) * NS * MR * kTileN);
    const uint32_t dst = map_to_rank(slot0, 0);
    const uint32_t rbar = map_to_rank(smem_u32(recv), 0);
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m) st_async_f32(dst + ((s * MR + m) * kTileN + c) * 4, vs[s][m], rbar);
    return;
  }
  if (p.split > 1) {
    if (!mbar_wait_cluster(recv, 0)) {
      if ((threadIdx.x & 31) == 0) record_fault(p.fault, kFaultFullWait);
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
  }

  if (p.kout > 1) {
    // Clusters of this tile meet in the workspace: every cluster stores its
    // partial sums, the last to arrive adds them in K order.
    float* ws = g_dp_ws[p.ws_slot] + static_cast<size_t>(tile) * p.kout * NS * MR * kTileN;
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m) __stcg(ws + ((blockIdx.z * NS + s) * MR + m) * kTileN + c, vs[s][m]);
    __threadfence();
    named_bar_sync(1, kTileN);
    int* last = reinterpret_cast<int*>(smem + L.xchg_off) + 4 * MR;
    if (c == 0) {
      const unsigned before = atomicAdd(&g_dp_cnt[p.ws_slot][tile], 1u);
      *last = before == static_cast<unsigned>(p.kout - 1);
      if (*last) g_dp_cnt[p.ws_slot][tile] = 0u;  // every arrival of this launch is in
    }
    named_bar_sync(1, kTileN);
    if (!*last) return;
    __threadfence();
    // The tile's kout x NS x MR x 128 partial sums come in with one bulk copy
    // over the used weight slots (one L2 round trip instead of one per part),
    // then each thread adds its column's parts in K order from shared memory.
    const uint32_t wbytes = static_cast<uint32_t>(p.kout * NS * MR * kTileN * 4);
    const bool bulk = wbytes <= L.act_off;
    const float* src = ws;
    if (bulk) {
      float* wsm = reinterpret_cast<float*>(smem);
      if (c == 0) {
        fence_proxy_async_global();
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(abar, wbytes);
        bulk_load(wsm, ws, wbytes, abar);
      }
      if (!mbar_wait(abar, 1)) {
        if ((threadIdx.x & 31) == 0) record_fault(p.fault, kFaultFullWait);
        mbar_wait(abar, 1);  // the copy lands before the CTA may exit
      }
      src = wsm;
    }
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float v = bulk ? src[(s * MR + m) * kTileN + c] : __ldcg(src + (s * MR + m) * kTileN + c);
        for (int k = 1; k < p.kout; ++k) {
          const float* q = src + ((k * NS + s) * MR + m) * kTileN + c;
          v = __fadd_rn(v, bulk ? *q : __ldcg(q));
        }
        vs[s][m] = v;
      }
  }

  // ---------------------------------------------------------------- epilogue (threads 0..127 of one rank 0)
  if (threadIdx.x == 0) QLIN_TL(p, 6);
  const int q4 = threadIdx.x >> 5;
  const bool valid = en < S0.n;
  if (EPI == kEpiOut) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    if (p.peer.tx[0]) {
      // Column-split layer: every row also goes to every rank's exchange
      // buffer, four columns (two flagged words) per store from lanes 4j.
      const DpPeer& pr = p.peer;
      const unsigned seq = pr.tx_state[0] + 1u;
      const unsigned long long tag = static_cast<unsigned long long>(seq) << 32;
      const long long obase = static_cast<long long>(seq & 1u) * pr.world * pr.tx_slot + pr.rank * pr.tx_slot;
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const bool sto = valid && m < p.M;
        float v = vs[0][m];
        if (WB == 8) v = __fmul_rn(v, pre_s0);
        const __nv_bfloat16 bv = __float2bfloat16_rn(v);
        if (sto) out[static_cast<long long>(m) * p.ldo + S0.out_col + en] = bv;
        const unsigned b0 = sto ? static_cast<unsigned>(__bfloat16_as_ushort(bv)) : 0u;
        const unsigned b1 = __shfl_down_sync(0xffffffffu, b0, 1);
        const unsigned b2 = __shfl_down_sync(0xffffffffu, b0, 2);
        const unsigned b3 = __shfl_down_sync(0xffffffffu, b0, 3);
        if (sto && (c & 3) == 0) {
          const long long e = obase + (static_cast<long long>(m) * (S0.n / 4) + en / 4) * 16;
          for (int q = 0; q < pr.world; ++q) st_sys_v2(pr.tx[q] + e, tag | (b0 | (b1 << 16)), tag | (b2 | (b3 << 16)));
        }
      }
    } else {
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (!valid || m >= p.M) continue;
        float v = vs[0][m];
        if (WB == 8) v = __fmul_rn(v, pre_s0);  // out * bs (kernels/gemm.py:51-52)
        if (p.res) v = __fadd_rn(v, pre_res[m]);
        out[static_cast<long long>(m) * p.ldo + S0.out_col + en] = __float2bfloat16_rn(v);
      }
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
        if (valid && m < p.M)
          reinterpret_cast<__nv_bfloat16*>(p.out)[static_cast<long long>(m) * p.ldo + en] = __float2bfloat16_rn(h);
      } else {
        // kernels/gemm.py:198-211: round through bf16, per-64 amax, int8 codes
        hb[m] = bf16_round_f32(h);
        amax[m] = fabsf(hb[m]);
      }
    }
    if (EPI == kEpiSiluQuant) {
      // every row's warp amax first, one exchange with the other warp of each
      // 64-column group for all rows, then the codes
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int m = 0; m < MR; ++m) amax[m] = fmaxf(amax[m], __shfl_xor_sync(0xffffffffu, amax[m], o));
      if ((threadIdx.x & 31) == 0)
#pragma unroll
        for (int m = 0; m < MR; ++m) xchg[q4 * MR + m] = amax[m];
      named_bar_sync(2, kTileN);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float am = fmaxf(amax[m], xchg[(q4 ^ 1) * MR + m]);  // the other warp of this 64-column group
        const float scq = fmaxf(__fdiv_rn(am, 127.0f), 1e-8f);
        const int8_t qv = round_i8(__fdiv_rn(hb[m], scq));
        if (valid && m < p.M) {
          p.out_q[static_cast<long long>(m) * p.n_q + en] = qv;
          if ((c & 63) == 0) p.out_s[static_cast<long long>(m) * (p.n_q / 64) + en / 64] = scq;
        }
      }
    }
  }
  if (threadIdx.x == 0) QLIN_TL(p, 7);
}

}  // namespace qlin
