// Decode-step neighbours of the quantised-linear path: the kernels between
// the projections of one decode step of the hybrid stack (the reference's
// kernels/attention.py and kernels/linear_attn.py at one new token per
// candidate).  All are HBM- or latency-bound: they move the KV cache, the
// delta-rule state and a few activation rows.
//
//   qk_norm_rope_kernel   q/k RMSNorm (1 + w), partial rotate-half RoPE, and
//                         the K/V cache write (bf16, or int8 with one fp32
//                         amax/127 scale per (position, head, side))
//   attn_decode_kernel    single-query attention over the cache, GQA heads of
//                         one KV head together, positions split over the CTAs
//                         of a thread-block cluster, combined through
//                         distributed shared memory (no global scratch)
//   delta_decode_kernel   gated delta-rule recurrent update of the fp32 state
//   conv_silu_kernel      depthwise causal conv (width 4) + SiLU
//   conv_state_update_kernel   the conv window shift
//
// fp32 arithmetic follows the reference's order per element; reductions
// (sums of squares, dot products, the softmax) are this file's own order.
// Positions may come from device memory (`pos_dev`) so that a decode step can
// be captured once in a CUDA graph and replayed at every position.
#pragma once

#include "producers.cuh"
#include "qlin_common.cuh"

namespace qlin {

constexpr int kDecThreads = 256;

// E consecutive bf16 (E = 2, 4, 8) at p -> fp32.
template <int E>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float (&v)[E]) {
  if constexpr (E == 8) {
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(p), v);
  } else if constexpr (E == 4) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(r.x << 16);
    v[1] = __uint_as_float(r.x & 0xFFFF0000u);
    v[2] = __uint_as_float(r.y << 16);
    v[3] = __uint_as_float(r.y & 0xFFFF0000u);
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = __bfloat162float(p[j]);
  }
}

template <int E>
__device__ __forceinline__ void store_bf16(__nv_bfloat16* p, const float (&v)[E]) {
#pragma unroll
  for (int j = 0; j < E; ++j) p[j] = __float2bfloat16_rn(v[j]);
}

// E int8 at p -> fp32 (E = 4 or 8, naturally aligned).
template <int E>
__device__ __forceinline__ void load_i8(const int8_t* p, float (&v)[E]) {
  if constexpr (E == 8) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = static_cast<float>(static_cast<int8_t>(((j < 4 ? r.x : r.y) >> (8 * (j & 3))) & 0xFF));
  } else {
    const uint32_t r = *reinterpret_cast<const uint32_t*>(p);
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = static_cast<float>(static_cast<int8_t>((r >> (8 * j)) & 0xFF));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------- qk_norm_rope
struct QkRopeArgs {
  const __nv_bfloat16* proj;  // [T, ldp]: per q head hd query + hd gate dims, then k heads, then v heads
  long long ldp;
  const __nv_bfloat16* qn;    // [hd]
  const __nv_bfloat16* kn;    // [hd]
  const float* invf;          // [rd / 2]
  __nv_bfloat16* qout;        // [T, nq * hd]
  void* kvc;                  // [rows, 2 * nkv * hd] bf16 or int8
  float* kvs;                 // [rows, 2 * nkv] (int8 cache)
  const int* pos_dev;         // position from device memory, or null
  long long kv_stride, kvs_stride;  // per-row cache slice (batch mode), elements
  int T, nq, nkv, rd, pos0, batch;
  float eps;
};

// kernels/attention.py:20-133.  One warp per (row, head); lane l owns dims
// [l*E, (l+1)*E).  Head index hi < nq: q head; < nq + nkv: k head; else v head.
template <int HD, bool INT8>
__global__ void __launch_bounds__(kDecThreads) qk_norm_rope_kernel(const __grid_constant__ QkRopeArgs a) {
  constexpr int E = HD / 32;
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nh = a.nq + 2 * a.nkv;
  const long long item = static_cast<long long>(blockIdx.x) * (kDecThreads / 32) + warp;
  if (item >= static_cast<long long>(a.T) * nh) return;
  const int row = static_cast<int>(item / nh), hi = static_cast<int>(item % nh);
  const int sns = 2 * a.nkv;
  float w[E];
  const bool vhead = hi >= a.nq + a.nkv;
  if (!vhead) {
    load_bf16<E>((hi < a.nq ? a.qn : a.kn) + lane * E, w);
#pragma unroll
    for (int j = 0; j < E; ++j) w[j] = __fadd_rn(w[j], 1.0f);
  }
  pdl_wait();
  const int base_pos = a.pos_dev ? *a.pos_dev : a.pos0;
  const int pos = a.batch ? base_pos : base_pos + row;
  const __nv_bfloat16* src;
  if (hi < a.nq) src = a.proj + row * a.ldp + hi * 2 * HD;
  else if (!vhead) src = a.proj + row * a.ldp + a.nq * 2 * HD + (hi - a.nq) * HD;
  else src = a.proj + row * a.ldp + a.nq * 2 * HD + a.nkv * HD + (hi - a.nq - a.nkv) * HD;
  float x[E];
  load_bf16<E>(src + lane * E, x);
  const long long kv_row = (a.batch ? row * a.kv_stride : 0) + static_cast<long long>(pos) * sns * HD;
  const long long kvs_row = (a.batch ? row * a.kvs_stride : 0) + static_cast<long long>(pos) * sns;
  float y[E];
  if (vhead) {
#pragma unroll
    for (int j = 0; j < E; ++j) y[j] = x[j];
  } else {
    // RMSNorm (1 + w) over HD (attention.py:45-50)
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss = __fadd_rn(ss, __fmul_rn(x[j], x[j]));
    const float rstd = rsqrt_ieee(__fadd_rn(__fdiv_rn(warp_sum(ss), static_cast<float>(HD)), a.eps));
    float yn[E];
#pragma unroll
    for (int j = 0; j < E; ++j) yn[j] = __fmul_rn(__fmul_rn(x[j], rstd), w[j]);
    // rotate-half RoPE on dims < rd; the partner of dim d < rd/2 is d + rd/2
    const int d2 = a.rd / 2;
    const int step = d2 / E;  // lanes between partners
    const int partner = lane < step ? lane + step : lane - step;
    const float scale = hi < a.nq ? __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(HD))) : 1.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float other = __shfl_sync(0xffffffffu, yn[j], partner);
      const int d = lane * E + j;
      if (d < a.rd) {
        const bool lo = d < d2;
        const float th = __fmul_rn(static_cast<float>(pos), a.invf[lo ? d : d - d2]);
        const float c = cosf(th), s = sinf(th);
        // plo = ylo cos - yhi sin; phi = yhi cos + ylo sin (attention.py:52-54)
        const float r = lo ? __fsub_rn(__fmul_rn(yn[j], c), __fmul_rn(other, s))
                           : __fadd_rn(__fmul_rn(yn[j], c), __fmul_rn(other, s));
        y[j] = __fmul_rn(r, scale);
      } else {
        y[j] = __fmul_rn(yn[j], scale);
      }
    }
  }
  if (hi < a.nq) {
    store_bf16<E>(a.qout + static_cast<long long>(row) * a.nq * HD + hi * HD + lane * E, y);
    return;
  }
  const int col = vhead ? (a.nkv + hi - a.nq - a.nkv) : (hi - a.nq);  // head slot in the cache row
  if constexpr (INT8) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) amax = fmaxf(amax, fabsf(y[j]));
    amax = warp_max(amax);
    const float sc = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    int8_t* dst = static_cast<int8_t*>(a.kvc) + kv_row + col * HD + lane * E;
#pragma unroll
    for (int j = 0; j < E; ++j) dst[j] = round_i8(__fdiv_rn(y[j], sc));
    if (lane == 0) a.kvs[kvs_row + col] = sc;
  } else {
    store_bf16<E>(static_cast<__nv_bfloat16*>(a.kvc) + kv_row + col * HD + lane * E, y);
  }
}

// ---------------------------------------------------------------- attn_decode
struct AttnDecodeArgs {
  const __nv_bfloat16* q;  // [B, nq * hd] (already scaled by 1/sqrt(hd))
  const void* kvc;         // [rows, 2 * nkv * hd]; candidate b's rows start at b * kv_stride
  const float* kvs;        // [rows, 2 * nkv] (int8 cache)
  __nv_bfloat16* out;      // [B, nq * hd]
  const int* pos_dev;      // last position (inclusive) from device memory, or null
  long long kv_stride, kvs_stride;
  int pos, nq, nkv;
  int hsplit;              // CTAs per KV head, each serving G of its query heads
};

// Per-warp online-softmax state of the G query heads of one KV head.
template <int G, int E>
struct SoftmaxState {
  float m[G], l[G], acc[G][E];
};

// Raw cache words of one lane: NWD 32-bit words, loaded in one access.
template <int NWD>
__device__ __forceinline__ void load_words(const void* p, uint32_t (&w)[NWD]) {
  if constexpr (NWD == 4) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    w[0] = r.x, w[1] = r.y, w[2] = r.z, w[3] = r.w;
  } else if constexpr (NWD == 2) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    w[0] = r.x, w[1] = r.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}
// element j of raw words: int8 (4 per word) or bf16 (2 per word) -> fp32
template <bool INT8, int NWD>
__device__ __forceinline__ float raw_elem(const uint32_t (&w)[NWD], int j) {
  if constexpr (INT8) return static_cast<float>(static_cast<int8_t>((w[j >> 2] >> (8 * (j & 3))) & 0xFF));
  return __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16));
}

// kernels/attention.py:209-267.  Cluster of S CTAs per (KV head, group of G of
// its query heads, candidate) -- a KV head's query heads may be split over
// `hsplit` CTA groups that read the same cache rows, for more CTAs:
// rank r covers positions [r n / S, (r+1) n / S) of the n = pos + 1; warp w of
// a CTA the positions w, w + 8, ... of that range, CH at a time: the chunk's
// K/V rows are all requested before any is used (one memory latency per
// chunk, not per position), then per query head the CH scores (lane partial
// dots, warp sums interleaved), and one online-softmax update per chunk:
//   m' = max(m, max_c s_c);  l = l e^{m - m'} + sum_c e^{s_c - m'};
//   acc = acc e^{m - m'} + sum_c e^{s_c - m'} v_c.
// The warps' states merge in shared memory; every rank > 0 then stores its
// merged state into its slot of rank 0's shared memory (remote stores, one
// cluster barrier with release / acquire), and rank 0 merges the ranks in
// rank order from its own shared memory, then out = acc / l.
constexpr int kAdMaxRanks = 8;
template <int G, int E, bool INT8>
__global__ void __launch_bounds__(kDecThreads) attn_decode_kernel(const __grid_constant__ AttnDecodeArgs a) {
  constexpr int HD = 32 * E;
  constexpr int NW = kDecThreads / 32;
  // per-warp m, l [NW][G] and acc [NW][G][HD]; then the CTA's merged m, l [G]
  // (acc merged into warp 0's slot).  Rank 0 reads the other ranks' merged
  // state through distributed shared memory.
  extern __shared__ __align__(16) float sm[];
  float* sm_m = sm;
  float* sm_l = sm + NW * G;
  float* sm_acc = sm + 2 * NW * G;
  float* fm = sm_acc + NW * G * HD;
  float* fl = fm + G;
  float* xs = fl + G;  // rank 0: slot r - 1 holds rank r's merged acc [G * HD], m [G], l [G]
  constexpr int kSlot = G * HD + 2 * G;
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = static_cast<int>(gridDim.x);
  const int rank = static_cast<int>(blockIdx.x);
  const int kvh = blockIdx.y / a.hsplit, b = blockIdx.z;
  const int h0 = kvh * G * a.hsplit + (blockIdx.y % a.hsplit) * G;  // first query head of this CTA
  pdl_wait();
  const int n = (a.pos_dev ? *a.pos_dev : a.pos) + 1;
  const int p0 = static_cast<int>(static_cast<long long>(rank) * n / S);
  const int p1 = static_cast<int>(static_cast<long long>(rank + 1) * n / S);
  const int sns = 2 * a.nkv;
  float q[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g)
    load_bf16<E>(a.q + static_cast<long long>(b) * a.nq * HD + (h0 + g) * HD + lane * E, q[g]);
  SoftmaxState<G, E> st;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    st.m[g] = -INFINITY;
    st.l[g] = 0.0f;
#pragma unroll
    for (int j = 0; j < E; ++j) st.acc[g][j] = 0.0f;
  }
  const long long kb = b * a.kv_stride, sb = b * a.kvs_stride;
  constexpr int CH = (INT8 && G <= 4) ? 8 : 4;   // positions per chunk of a warp (register budget)
  constexpr int NWD = INT8 ? E / 4 : E / 2;       // raw 32-bit words per lane and row
  constexpr int EB = INT8 ? 1 : 2;                // bytes per cache element
  const uint8_t* kvb = static_cast<const uint8_t*>(a.kvc);
  for (int base = p0 + warp; base < p1; base += NW * CH) {
    uint32_t kr[CH][NWD], vr[CH][NWD];
    float ksc[CH], vsc[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int p = base + c * NW;
      if (p < p1) {
        const long long rowk = (kb + static_cast<long long>(p) * sns * HD) * EB;
        load_words<NWD>(kvb + rowk + (kvh * HD + lane * E) * EB, kr[c]);
        load_words<NWD>(kvb + rowk + ((a.nkv + kvh) * HD + lane * E) * EB, vr[c]);
        if constexpr (INT8) {
          ksc[c] = a.kvs[sb + static_cast<long long>(p) * sns + kvh];
          vsc[c] = a.kvs[sb + static_cast<long long>(p) * sns + a.nkv + kvh];
        } else {
          ksc[c] = vsc[c] = 1.0f;
        }
      } else {
#pragma unroll
        for (int w = 0; w < NWD; ++w) kr[c][w] = vr[c][w] = 0u;
        ksc[c] = vsc[c] = 0.0f;
      }
    }
    float sc[G][CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      float k[E];
#pragma unroll
      for (int j = 0; j < E; ++j) {
        k[j] = raw_elem<INT8, NWD>(kr[c], j);
        if constexpr (INT8) k[j] = __fmul_rn(k[j], ksc[c]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float d = 0.0f;
#pragma unroll
        for (int j = 0; j < E; ++j) d = __fadd_rn(d, __fmul_rn(q[g][j], k[j]));
        sc[g][c] = d;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < CH; ++c) sc[g][c] = __fadd_rn(sc[g][c], __shfl_xor_sync(0xffffffffu, sc[g][c], o));
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mc = sc[g][0];  // position base < p1 always
#pragma unroll
      for (int c = 1; c < CH; ++c)
        if (base + c * NW < p1) mc = fmaxf(mc, sc[g][c]);
      const float mn = fmaxf(st.m[g], mc);
      const float alpha = expf(st.m[g] - mn);  // 0 for the first chunk (m = -inf)
      float pe[CH];
      float ps = 0.0f;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        pe[c] = base + c * NW < p1 ? expf(sc[g][c] - mn) : 0.0f;
        ps = __fadd_rn(ps, pe[c]);
      }
      st.l[g] = __fadd_rn(__fmul_rn(st.l[g], alpha), ps);
#pragma unroll
      for (int j = 0; j < E; ++j) {
        float t = __fmul_rn(st.acc[g][j], alpha);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          float v = raw_elem<INT8, NWD>(vr[c], j);
          if constexpr (INT8) v = __fmul_rn(v, vsc[c]);
          t = __fadd_rn(t, __fmul_rn(pe[c], v));
        }
        st.acc[g][j] = t;
      }
      st.m[g] = mn;
    }
  }
  // merge the warps of this CTA: every (g, d) by one thread, into warp 0's slot
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      sm_m[warp * G + g] = st.m[g];
      sm_l[warp * G + g] = st.l[g];
    }
#pragma unroll
    for (int j = 0; j < E; ++j) sm_acc[(warp * G + g) * HD + lane * E + j] = st.acc[g][j];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kDecThreads) {
    const int g = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w * G + g]);
    float acc = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w)
        acc = __fadd_rn(acc, __fmul_rn(sm_acc[(w * G + g) * HD + d], expf(sm_m[w * G + g] - M)));
    }
    sm_acc[g * HD + d] = acc;
  }
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w * G + g]);
    float L = 0.0f;
    if (M != -INFINITY)
      for (int w = 0; w < NW; ++w) L = __fadd_rn(L, __fmul_rn(sm_l[w * G + g], expf(sm_m[w * G + g] - M)));
    fm[g] = M;
    fl[g] = L;
  }
  __syncthreads();
  // ranks > 0: merged state -> their slot of rank 0's shared memory
  if (S > 1 && rank > 0) {
    const uint32_t slot = map_to_rank(smem_u32(xs + (rank - 1) * kSlot), 0);
    for (int idx = threadIdx.x; idx < G * HD; idx += kDecThreads) st_cluster_f32(slot + idx * 4, sm_acc[idx]);
    if (threadIdx.x < G) {
      st_cluster_f32(slot + (G * HD + threadIdx.x) * 4, fm[threadIdx.x]);
      st_cluster_f32(slot + (G * HD + G + threadIdx.x) * 4, fl[threadIdx.x]);
    }
  }
  if (S > 1) {
    cluster_arrive_release();
    cluster_wait();
  }
  // rank 0 merges the ranks' states in rank order, then divides
  if (rank == 0) {
    for (int idx = threadIdx.x; idx < G * HD; idx += kDecThreads) {
      const int g = idx / HD, d = idx % HD;
      float M = fm[g];
      for (int r = 1; r < S; ++r) M = fmaxf(M, xs[(r - 1) * kSlot + G * HD + g]);
      float acc = 0.0f, L = 0.0f;
      for (int r = 0; r < S; ++r) {
        const float* xr = xs + (r - 1) * kSlot;
        const float mr = r == 0 ? fm[g] : xr[G * HD + g];
        if (mr == -INFINITY) continue;  // a rank without positions
        const float f = expf(mr - M);
        const float lr = r == 0 ? fl[g] : xr[G * HD + G + g];
        const float ar = r == 0 ? sm_acc[idx] : xr[idx];
        L = __fadd_rn(L, __fmul_rn(lr, f));
        acc = __fadd_rn(acc, __fmul_rn(ar, f));
      }
      a.out[static_cast<long long>(b) * a.nq * HD + (h0 + g) * HD + d] = __float2bfloat16_rn(__fdiv_rn(acc, L));
    }
  }
}

__host__ __device__ constexpr int attn_decode_smem(int G, int E) {
  return (2 * (kDecThreads / 32) * G + (kDecThreads / 32) * G * 32 * E + 2 * G +
          (kAdMaxRanks - 1) * (G * 32 * E + 2 * G)) *
         4;
}

// ---------------------------------------------------------------- delta_decode
// kernels/linear_attn.py:172-207.  CTA = (head h, candidate b, 32-column
// slab); 4 warps x 32 lanes: lane = column c of the slab, warp w = rows
// [32 w, 32 w + 32) of the DK = 128 rows.
//   qn = q rsqrt(|q|^2 + 1e-6) / sqrt(DK);  kn = k rsqrt(|k|^2 + 1e-6)
//   S *= exp(g);  kv = kn^T S;  delta = (v - kv) beta;  S += kn delta^T;
//   out = qn^T S
constexpr int kDeltaDK = 128, kDeltaDV = 128, kDeltaRows = 32, kDeltaWarps = 4;
__global__ void __launch_bounds__(kDeltaWarps * 32) delta_decode_kernel(
    const __nv_bfloat16* __restrict__ qkv, long long ldq, const float* __restrict__ g, const float* __restrict__ beta,
    float* __restrict__ state, __nv_bfloat16* __restrict__ out, int nh) {
  __shared__ float qn_s[kDeltaDK], kn_s[kDeltaDK], part[kDeltaWarps][32], red[2][kDeltaWarps];
  pdl_launch_dependents();
  const int h = blockIdx.x, b = blockIdx.y, slab = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = slab * 32 + lane;
  float* S = state + (static_cast<long long>(b) * nh + h) * kDeltaDK * kDeltaDV;
  pdl_wait();  // the state is written by this layer's previous step, not a parameter
  float sv[kDeltaRows];
#pragma unroll
  for (int i = 0; i < kDeltaRows; ++i) sv[i] = S[static_cast<long long>(warp * kDeltaRows + i) * kDeltaDV + c];
  const __nv_bfloat16* row = qkv + static_cast<long long>(b) * ldq;
  const int t = threadIdx.x;  // 128 threads: one q and one k element each
  const float qv = __bfloat162float(row[h * kDeltaDK + t]);
  const float kv0 = __bfloat162float(row[nh * kDeltaDK + h * kDeltaDK + t]);
  const float vq = warp_sum(__fmul_rn(qv, qv)), vk = warp_sum(__fmul_rn(kv0, kv0));
  if (lane == 0) {
    red[0][warp] = vq;
    red[1][warp] = vk;
  }
  __syncthreads();
  float sq = 0.0f, sk = 0.0f;
#pragma unroll
  for (int w = 0; w < kDeltaWarps; ++w) {
    sq = __fadd_rn(sq, red[0][w]);
    sk = __fadd_rn(sk, red[1][w]);
  }
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(kDeltaDK)));
  qn_s[t] = __fmul_rn(__fmul_rn(qv, rsqrt_ieee(__fadd_rn(sq, 1e-6f))), inv);
  kn_s[t] = __fmul_rn(kv0, rsqrt_ieee(__fadd_rn(sk, 1e-6f)));
  const float eg = expf(g[static_cast<long long>(b) * nh + h]);
  const float bt = beta[static_cast<long long>(b) * nh + h];
  const float vv = __bfloat162float(row[2 * nh * kDeltaDK + h * kDeltaDV + c]);
  __syncthreads();
  float kvp = 0.0f;
#pragma unroll
  for (int i = 0; i < kDeltaRows; ++i) {
    sv[i] = __fmul_rn(sv[i], eg);
    kvp = __fadd_rn(kvp, __fmul_rn(kn_s[warp * kDeltaRows + i], sv[i]));
  }
  part[warp][lane] = kvp;
  __syncthreads();
  float kvs = 0.0f;
#pragma unroll
  for (int w = 0; w < kDeltaWarps; ++w) kvs = __fadd_rn(kvs, part[w][lane]);
  const float delta = __fmul_rn(__fsub_rn(vv, kvs), bt);
  __syncthreads();  // part is reused below
  float op = 0.0f;
#pragma unroll
  for (int i = 0; i < kDeltaRows; ++i) {
    sv[i] = __fadd_rn(sv[i], __fmul_rn(kn_s[warp * kDeltaRows + i], delta));
    op = __fadd_rn(op, __fmul_rn(qn_s[warp * kDeltaRows + i], sv[i]));
    S[static_cast<long long>(warp * kDeltaRows + i) * kDeltaDV + c] = sv[i];
  }
  part[warp][lane] = op;
  __syncthreads();
  if (warp == 0) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kDeltaWarps; ++w) o = __fadd_rn(o, part[w][lane]);
    out[static_cast<long long>(b) * nh * kDeltaDV + h * kDeltaDV + c] = __float2bfloat16_rn(o);
  }
}

// ---------------------------------------------------------------- conv
// kernels/linear_attn.py:10-47 (KS = 4).  Thread = 8 channels of one output
// row.  Sequence mode: tap j of row t reads input row t - 3 + j, or state row
// 3 + (t - 3 + j) before the first input row.  Batch mode: taps 0..2 read the
// row's own state rows 3 t + j, tap 3 its input row.
//   acc = sum_j x_j * w[:, j] (j ascending);  y = silu(acc)
constexpr int kConvKS = 4;
__global__ void __launch_bounds__(kDecThreads) conv_silu_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ state, __nv_bfloat16* __restrict__ y, int T, int C, int batch) {
  pdl_launch_dependents();
  const int t = blockIdx.y;
  const int c8 = blockIdx.x * kDecThreads + threadIdx.x;
  if (8 * c8 >= C) return;
  const int c0 = 8 * c8;
  float wv[8][kConvKS];
  {
    // w [C, 4] bf16: the 8 channels' 32 weights are contiguous
    const uint4* wp = reinterpret_cast<const uint4*>(w + static_cast<long long>(c0) * kConvKS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      bf16x8_to_f32(wp[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[2 * i + j / 4][j % 4] = f[j];
    }
  }
  pdl_wait();
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int j = 0; j < kConvKS; ++j) {
    const __nv_bfloat16* src;
    if (batch) {
      src = j < kConvKS - 1 ? state + (static_cast<long long>(t) * (kConvKS - 1) + j) * C + c0
                            : x + static_cast<long long>(t) * ldx + c0;
    } else {
      const int r = t - (kConvKS - 1) + j;
      src = r >= 0 ? x + static_cast<long long>(r) * ldx + c0 : state + static_cast<long long>(kConvKS - 1 + r) * C + c0;
    }
    float xv[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(src), xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(xv[i], wv[i][j]));
  }
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(acc[i], sigmoid_ref(acc[i]));
  store_bf16<8>(y + static_cast<long long>(t) * C + c0, o);
}

// kernels/linear_attn.py:50-83.  Thread = 8 channels of one state window
// (one candidate in batch mode).  Every value is read before any is written.
__global__ void __launch_bounds__(kDecThreads) conv_state_update_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, __nv_bfloat16* __restrict__ state, int T, int C, int batch) {
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int c8 = blockIdx.x * kDecThreads + threadIdx.x;
  if (8 * c8 >= C) return;
  const int c0 = 8 * c8;
  pdl_wait();
  constexpr int W = kConvKS - 1;
  uint4 v[W];
  __nv_bfloat16* st = state + static_cast<long long>(batch ? b * W : 0) * C + c0;
  if (batch) {
    v[0] = *reinterpret_cast<const uint4*>(st + C);
    v[1] = *reinterpret_cast<const uint4*>(st + 2 * C);
    v[2] = *reinterpret_cast<const uint4*>(x + static_cast<long long>(b) * ldx + c0);
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const int src = T - W + j;
      v[j] = src >= 0 ? *reinterpret_cast<const uint4*>(x + static_cast<long long>(src) * ldx + c0)
                      : *reinterpret_cast<const uint4*>(st + static_cast<long long>(src + W) * C);
    }
  }
#pragma unroll
  for (int j = 0; j < W; ++j) *reinterpret_cast<uint4*>(st + static_cast<long long>(j) * C) = v[j];
}

// conv_silu_kernel and conv_state_update_kernel of one decode step (batch
// mode, one new row per candidate) in one launch: thread = 8 channels of
// candidate b; it reads the candidate's 3 window rows and its input row,
// writes y as conv_silu does, then the shifted window as conv_state_update
// does.  No other thread touches these channels of this window.
__global__ void __launch_bounds__(kDecThreads) conv_silu_update_kernel(
    const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ state, __nv_bfloat16* __restrict__ y, int C) {
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int c8 = blockIdx.x * kDecThreads + threadIdx.x;
  if (8 * c8 >= C) return;
  const int c0 = 8 * c8;
  float wv[8][kConvKS];
  {
    const uint4* wp = reinterpret_cast<const uint4*>(w + static_cast<long long>(c0) * kConvKS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      bf16x8_to_f32(wp[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[2 * i + j / 4][j % 4] = f[j];
    }
  }
  pdl_wait();
  constexpr int W = kConvKS - 1;
  __nv_bfloat16* st = state + static_cast<long long>(b) * W * C + c0;
  uint4 raw[kConvKS];
#pragma unroll
  for (int j = 0; j < W; ++j) raw[j] = *reinterpret_cast<const uint4*>(st + static_cast<long long>(j) * C);
  raw[W] = *reinterpret_cast<const uint4*>(x + static_cast<long long>(b) * ldx + c0);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int j = 0; j < kConvKS; ++j) {
    float xv[8];
    bf16x8_to_f32(raw[j], xv);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(xv[i], wv[i][j]));
  }
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(acc[i], sigmoid_ref(acc[i]));
  store_bf16<8>(y + static_cast<long long>(b) * C + c0, o);
#pragma unroll
  for (int j = 0; j < W; ++j) *reinterpret_cast<uint4*>(st + static_cast<long long>(j) * C) = raw[j + 1];
}

}  // namespace qlin
