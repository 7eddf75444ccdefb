// Launch arguments shared by the small-M weight-streaming kernel
// (tcgemv.cuh) and the prefill GEMMs (tcgemm.cuh, tcgemm_w4.cuh).
//
// Every hot-path entry point maps onto one of three epilogues:
//   kEpiOut        gemm_i8 / gemm_w4 (+ residual) and proj3 / proj3_w4 (up to
//                  three column segments written side by side)
//   kEpiSiluBf16   mlp_gate_up        (two weight streams, bf16 h)
//   kEpiSiluQuant  mlp_gate_up_quant  / mlp_gate_up_quant_w4 (two weight
//                  streams, h rounded through bf16 and re-quantised per 64
//                  columns)
// Output columns are cut into 128-column tiles (128 bytes of one weight row:
// 128 int8 columns, or 128 packed W4 columns holding two K values each).
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kTileN = 128;

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
  CUtensorMap ta;    // activations a_q [M, K], 128-byte-swizzled boxes of 128 K x rows
  GemvSeg seg[3];    // kEpiOut: column segments; gate/up epilogues: seg[0]=gate, seg[1]=up
  int nseg;
  const int8_t* a_q;  // [M, K]
  const float* a_s;   // [M, K/64]
  int M, K, wgrp;
  int split;          // K ranges per tile == cluster size
  int bs;             // 64-K groups per batch (one barrier / commit per batch)
  int rb;             // batch slots in the weight ring
  int ab;             // W4: batch slots in the unpacked-weight ring
  int nbb;            // batch accumulators in tensor memory
  int gmax;           // max groups one CTA handles
  int part_alias;     // partial sums land in rank 0's (finished) MMA operand region
  void* out;          // bf16, row stride ldo
  long long ldo;
  const void* res;    // bf16 residual or null, row stride ldr
  long long ldr;
  int8_t* out_q;      // kEpiSiluQuant: int8 [M, n_q]
  float* out_s;       // kEpiSiluQuant: fp32 [M, n_q/64]
  int n_q;
  unsigned* fault;    // device fault word (bounded waits)
  int tl_slot;        // tuning builds: phase-timeline slot of this launch (-1: none)
  const void* peer;   // column-split layer: the dp kernel's DpPeer (host copy), or null
};

#ifdef QLIN_TUNING
// Phase timeline of the small-M kernel (tuning builds only): %globaltimer
// stamps per CTA and launch slot, read back with qlin_debug_timeline.
constexpr int kTlSlots = 16, kTlCtas = 2048, kTlStamps = 8;
__device__ unsigned long long g_qlin_tl[kTlSlots][kTlCtas][kTlStamps];
#define QLIN_TL(args, k)                                                                          \
  do {                                                                                            \
    if ((args).tl_slot >= 0) {                                                                    \
      const unsigned cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);       \
      if (cta_ < kTlCtas) g_qlin_tl[(args).tl_slot][cta_][k] = global_ns();                      \
    }                                                                                             \
  } while (0)
#else
#define QLIN_TL(args, k) \
  do {                   \
  } while (0)
#endif

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

}  // namespace qlin
