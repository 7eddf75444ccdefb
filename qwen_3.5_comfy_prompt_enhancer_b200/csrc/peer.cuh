// All-gathers over NVLink peer memory for the column-split layer.
//
// peer_allgather_kernel (arrival counters).  Every rank owns a gather buffer
// and an arrival array of `world` 32-bit counters, both opened by every
// other rank through CUDA IPC (no multicast objects).  One launch on rank r:
//   1. every CTA copies its slice of r's shard into r's slot of every rank's
//      gather buffer -- its own included -- over NVLink;
//   2. each CTA then adds 1 to arrival[r] on every rank (release, system
//      scope, after one system-scope fence);
//   3. CTA 0 waits until its own arrival[q] has reached expected[q] +
//      gridDim.x for every rank q, then advances expected (device memory, so
//      the kernel also works inside CUDA-graph replays).  The wait is
//      time-bounded: past the limit it records a fault and returns (the
//      context stays usable).
// Counters only grow, so no reset is ever needed.
//
// peer_ll_gather_kernel (flagged words, below) is the lower-latency form the
// column-split layer uses.
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kPeerMax = 8;
constexpr int kPeerThreads = 256;
constexpr int kPeerMaxParts = 2;
constexpr int kPeerMaxCtas = 64;

struct PeerPart {
  const uint8_t* src;    // this rank's part: rows x row_bytes, row stride src_ld
  long long src_ld;
  long long rows, row_bytes;
  long long dst_off;     // byte offset of rank 0's slot in every gather buffer
  long long dst_ld;      // row stride of the slots (bytes)
  int unit;              // 16 or 4: bytes per copy (every size, stride and address a multiple)
};

struct PeerGatherArgs {
  uint8_t* bufs[kPeerMax];        // every rank's gather buffer (peer pointers; own at [rank])
  unsigned* arrive[kPeerMax];     // every rank's arrival counters (peer pointers)
  unsigned* expected;             // this rank's expected counts [world]
  PeerPart part[kPeerMaxParts];
  int nparts;
  int world, rank;
  unsigned* fault;
};

__device__ __forceinline__ void st_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__device__ __forceinline__ void peer_copy_part(const PeerGatherArgs& a, const PeerPart& p) {
  const long long per_row = p.row_bytes / static_cast<long long>(sizeof(T));
  const long long n = p.rows * per_row;
  const long long slot = p.dst_off + static_cast<long long>(a.rank) * p.row_bytes;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / per_row, c = i - row * per_row;
    const T v = *reinterpret_cast<const T*>(p.src + row * p.src_ld + c * sizeof(T));
    const long long d = slot + row * p.dst_ld + c * sizeof(T);
    for (int q = 0; q < a.world; ++q) *reinterpret_cast<T*>(a.bufs[q] + d) = v;
  }
}

__global__ void __launch_bounds__(kPeerThreads) peer_allgather_kernel(const __grid_constant__ PeerGatherArgs a) {
  // The next launch may be placed now; the parts are read only once the
  // preceding kernel (their producer) has completed.
  pdl_launch_dependents();
  pdl_wait();
  // 1. my parts -> my slot of every rank's buffer
  for (int pi = 0; pi < a.nparts; ++pi) {
    if (a.part[pi].unit == 16) peer_copy_part<uint4>(a, a.part[pi]);
    else peer_copy_part<uint32_t>(a, a.part[pi]);
  }
  // 2. announce this CTA's part on every rank: the CTA barrier orders every
  // thread's stores before the signalling thread's system-scope release
  // (cumulativity), so one fence per signal, not one per thread
  __syncthreads();
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys_add(a.arrive[threadIdx.x] + a.rank, 1u);
  }
  if (blockIdx.x != 0) return;
  // 3. wait for every rank's parts of this call
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < a.world) {
    const unsigned want = a.expected[threadIdx.x] + gridDim.x;
    const unsigned* mine = a.arrive[a.rank] + threadIdx.x;
    const unsigned long long t0 = global_ns();
    // counters wrap after 2^32 parts; the signed difference stays valid.
    // Relaxed polling, then one system-scope fence: the acquire side of the
    // peers' release.
    while (static_cast<int>(ld_relaxed_sys(mine) - want) < 0) {
      if (global_ns() - t0 > wait_limit_ns()) {
        failed = 1;
        break;
      }
    }
    __threadfence_system();
  }
  __syncthreads();
  if (threadIdx.x == 0 && failed) record_fault(a.fault, kFaultFullWait);
  // advance the expected counts (only this CTA reads them)
  if (threadIdx.x < a.world) a.expected[threadIdx.x] += gridDim.x;
}

// ---------------------------------------------------------------- flagged-word all-gather
// The column-split layer's gathers are a few KB to a few MB per rank and sit
// between two dependent kernels, so their latency, not their bandwidth, is
// what the layer pays.  The arrival-counter protocol above needs a
// system-scope fence after the NVLink stores (a round trip to every peer)
// before the release, and an acquire on the waiting side.  This protocol
// needs neither: every 8-byte word a rank sends carries the call's sequence
// number in its high half, so a receiver that reads a word with the current
// sequence number holds valid data (a naturally aligned 64-bit access is
// single-copy atomic, and each word is checked on its own).
//
// Exchange buffer of every rank (zero once): [2 parities][world senders]
// [slot_bytes]; call number s uses parity s & 1.  A sender's slot holds its
// parts one after the other, each padded to 16 bytes, as words
// (seq << 32 | 4 data bytes): two words per 8 data bytes (unit 8, one 16-byte
// store) or one word per 4 data bytes (unit 4).  One launch on rank r:
//   1. for every unit of r's parts: copy it into r's slot of `dst` and store
//      its words into r's slot of every other rank's exchange buffer;
//   2. for every unit of every other rank q: poll own exchange buffer until
//      the words carry this call's sequence number (bounded), then write the
//      data into q's slot of `dst`;
//   3. the last CTA to finish advances the sequence number in `state`.
// Two parities suffice: rank r's call s + 2 starts after its call s + 1 has
// received every rank's call-(s + 1) words, which every rank sends only once
// its own call s (and so its reads of parity s & 1) has completed.
constexpr int kLlMaxParts = 4;
constexpr int kLlBatch = 4;  // words a receiving thread keeps in flight

struct LlPart {
  const uint8_t* src;    // this rank's block: rows x row_bytes, row stride src_ld
  long long src_ld;
  long long rows, row_bytes;
  long long dst_off, dst_ld;   // rank q's block at dst + dst_off + q * row_bytes, rows dst_ld apart
  long long ll_off;      // byte offset of the part's words in a sender slot (multiple of 16)
  long long first;       // index of the part's first unit among all parts' units
  int unit;              // data bytes per unit: 8 or 4
};

struct LlGatherArgs {
  uint8_t* ll[kPeerMax];   // every rank's exchange buffer (peer pointers; own at [rank])
  long long slot_bytes;    // bytes of one sender slot
  unsigned* state;         // [0] sequence number of the last call, [1] completion counter
  LlPart part[kLlMaxParts];
  int nparts;
  long long units;         // all parts' units
  uint8_t* dst;            // this rank's destination
  int world, rank;
  // 0: the full gather; 1: send only (every rank's exchange, this rank's own
  // included; nothing advanced); 2: receive only (from every rank, own
  // included; advances `state` and, if set, adds one to state2[0])
  int mode;
  unsigned* state2;
  unsigned* fault;
};

__device__ __forceinline__ int ll_part_of(const LlGatherArgs& a, long long u) {
  int p = 0;
  while (p + 1 < a.nparts && u >= a.part[p + 1].first) ++p;
  return p;
}

__global__ void __launch_bounds__(kPeerThreads) peer_ll_gather_kernel(const __grid_constant__ LlGatherArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned seq = a.state[0] + 1u;
  const long long par = static_cast<long long>(seq & 1u) * a.world * a.slot_bytes;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const unsigned long long tag = static_cast<unsigned long long>(seq) << 32;
  // 1. send
  for (long long u = tid; a.mode != 2 && u < a.units; u += stride) {
    const LlPart& p = a.part[ll_part_of(a, u)];
    const long long v = u - p.first, per_row = p.row_bytes / p.unit;
    const long long row = v / per_row, c = (v - row * per_row) * p.unit;
    const uint8_t* s = p.src + row * p.src_ld + c;
    uint8_t* d = a.dst + p.dst_off + a.rank * p.row_bytes + row * p.dst_ld + c;
    const long long e = par + a.rank * a.slot_bytes + p.ll_off + v * 2 * p.unit;
    if (p.unit == 8) {
      const uint2 x = *reinterpret_cast<const uint2*>(s);
      if (a.mode == 0) *reinterpret_cast<uint2*>(d) = x;
      for (int q = 0; q < a.world; ++q)
        if (a.mode == 1 || q != a.rank) st_sys_v2(a.ll[q] + e, tag | x.x, tag | x.y);
    } else {
      const uint32_t x = *reinterpret_cast<const uint32_t*>(s);
      if (a.mode == 0) *reinterpret_cast<uint32_t*>(d) = x;
      for (int q = 0; q < a.world; ++q)
        if (a.mode == 1 || q != a.rank) st_sys_u64(a.ll[q] + e, tag | x);
    }
  }
  // 2. receive
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  bool dead = false;
  const unsigned long long t0 = global_ns();
  const long long total = a.mode == 1 ? 0 : static_cast<long long>(a.mode == 2 ? a.world : a.world - 1) * a.units;
  // kLlBatch words per thread in flight: their loads go out together, and a
  // word is polled again only while it is stale
  for (long long i0 = tid; i0 < total && !dead; i0 += stride * kLlBatch) {
    const uint8_t* w[kLlBatch];
    uint8_t* d[kLlBatch];
    bool need[kLlBatch];
    bool wide[kLlBatch];
#pragma unroll
    for (int b = 0; b < kLlBatch; ++b) {
      const long long i = i0 + b * stride;
      need[b] = i < total;
      w[b] = nullptr;
      d[b] = nullptr;
      wide[b] = false;
      if (!need[b]) continue;
      const long long qi = i / a.units, u = i - qi * a.units;
      const int q = (a.mode == 2 || static_cast<int>(qi) < a.rank) ? static_cast<int>(qi) : static_cast<int>(qi) + 1;
      const LlPart& p = a.part[ll_part_of(a, u)];
      const long long v = u - p.first, per_row = p.row_bytes / p.unit;
      const long long row = v / per_row, c = (v - row * per_row) * p.unit;
      w[b] = a.ll[a.rank] + par + q * a.slot_bytes + p.ll_off + v * 2 * p.unit;
      d[b] = a.dst + p.dst_off + q * p.row_bytes + row * p.dst_ld + c;
      wide[b] = p.unit == 8;
    }
    unsigned spin = 0;
    for (;;) {
      bool pending = false;
#pragma unroll
      for (int b = 0; b < kLlBatch; ++b) {
        if (!need[b]) continue;
        if (wide[b]) {
          unsigned long long w0, w1;
          ld_sys_v2(w[b], w0, w1);
          if (ll_fresh(w0, seq) && ll_fresh(w1, seq)) {
            *reinterpret_cast<uint2*>(d[b]) = make_uint2(static_cast<unsigned>(w0), static_cast<unsigned>(w1));
            need[b] = false;
          } else {
            pending = true;
          }
        } else {
          const unsigned long long w0 = ld_sys_u64(w[b]);
          if (ll_fresh(w0, seq)) {
            *reinterpret_cast<uint32_t*>(d[b]) = static_cast<unsigned>(w0);
            need[b] = false;
          } else {
            pending = true;
          }
        }
      }
      if (!pending) break;
      if ((++spin & 63u) == 0 && global_ns() - t0 > wait_limit_ns()) {
        dead = true;
        break;
      }
    }
  }
  if (dead) failed = 1;
  __syncthreads();
  if (threadIdx.x == 0 && failed) record_fault(a.fault, kFaultFullWait);
  // 3. the last CTA advances the sequence number (every CTA has read it)
  __shared__ unsigned last;
  if (threadIdx.x == 0) last = atomicAdd(a.state + 1, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (last && threadIdx.x == 0) {
    if (a.mode != 1) a.state[0] = seq;
    if (a.mode == 2 && a.state2) a.state2[0] += 1u;
    a.state[1] = 0u;
  }
}

}  // namespace qlin
