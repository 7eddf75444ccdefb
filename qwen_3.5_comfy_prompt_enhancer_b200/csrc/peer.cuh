// All-gather over NVLink peer memory for the column-split layer.
//
// Every rank owns a gather buffer and an arrival array of `world` 32-bit
// counters, both opened by every other rank through CUDA IPC (no multicast
// objects).  One launch of peer_allgather_kernel on rank r:
//   1. every CTA copies its slice of r's parts into r's slot of every rank's
//      gather buffer -- its own included -- over NVLink.  A part is a 2-D
//      block (rows x row_bytes, source row stride src_ld); rank r's slot
//      starts at dst_off + r * row_bytes with row stride dst_ld, so a shard of
//      output COLUMNS lands directly in its column range of every rank's
//      [rows, world * row_bytes] matrix (a 1-D shard is one row);
//   2. each CTA then fences at system scope and adds 1 to arrival[r] on every
//      rank (release, system scope);
//   3. the waiting CTAs (CTA 0, or every CTA when the gathered bytes are also
//      copied out) wait until their own arrival[q] has reached expected[q] +
//      gridDim.x for every rank q (acquire).  expected lives in device memory
//      and advances by gridDim.x per call, so the kernel also works inside
//      CUDA-graph replays; when every CTA waits, the last one to finish (a
//      completion counter) advances it, after all CTAs have read it.  The wait
//      is time-bounded: past the limit it records a fault and returns (the
//      context stays usable).
//   4. optionally every CTA then copies its slice of the local gather buffer
//      to `dst`.
// Counters only grow, so no reset is ever needed.  A buffer is not rewritten
// while a peer may still read it: the layer calls the gather twice per
// forward (h, then the output), and a rank's second gather cannot complete
// before every rank has finished the work between the two.
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
  unsigned* expected;             // this rank's expected counts [world] (+ a completion counter at [kPeerMax])
  PeerPart part[kPeerMaxParts];
  int nparts;
  uint8_t* dst;                   // optional: local gathered bytes [0, dst_bytes) copied here
  long long dst_bytes;            // multiple of 16
  int all_wait;                   // every CTA waits (needed for the copy to dst)
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
  if (!a.all_wait && blockIdx.x != 0) return;
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
  // 4. copy the gathered bytes out
  if (a.dst) {
    const long long n16 = a.dst_bytes / 16;
    const uint4* s = reinterpret_cast<const uint4*>(a.bufs[a.rank]);
    uint4* d = reinterpret_cast<uint4*>(a.dst);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
      d[i] = s[i];
  }
  // advance the expected counts once every waiting CTA has read them
  if (!a.all_wait) {
    if (threadIdx.x < a.world) a.expected[threadIdx.x] += gridDim.x;
    return;
  }
  __syncthreads();
  __shared__ unsigned last;
  if (threadIdx.x == 0) last = atomicAdd(a.expected + kPeerMax, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (last) {
    if (threadIdx.x < a.world) a.expected[threadIdx.x] += gridDim.x;
    if (threadIdx.x == 0) a.expected[kPeerMax] = 0;
  }
}

}  // namespace qlin
