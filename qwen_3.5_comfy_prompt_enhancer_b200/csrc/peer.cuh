// All-gather over NVLink peer memory for the column-split layer.
//
// Every rank owns a "gather" buffer of world x shard_bytes bytes and an
// arrival array of `world` 32-bit counters, both opened by every other rank
// through CUDA IPC (no multicast objects).  One launch of
// peer_allgather_kernel on rank r:
//   1. every CTA copies its slice of r's shard (16-byte stores) into slot r of
//      every rank's gather buffer -- its own included -- over NVLink;
//   2. each CTA then fences at system scope and adds 1 to arrival[r] on every
//      rank (release, system scope);
//   3. CTA 0 waits until its own arrival[q] has reached expected[q] for every
//      rank q (acquire), where expected advances by gridDim.x per call and
//      lives in device memory, so the kernel also works inside CUDA-graph
//      replays.  The wait is time-bounded: past the limit it sets the fault
//      word and returns (the context stays usable).
// Counters only grow, so no reset is ever needed.  A buffer is not rewritten
// while a peer may still read it: the layer calls the gather twice per
// forward (h, then the output), and a rank's second gather cannot complete
// before every rank has finished the work between the two.
#pragma once

#include "qlin_common.cuh"

namespace qlin {

constexpr int kPeerMax = 8;
constexpr int kPeerThreads = 256;

struct PeerGatherArgs {
  uint8_t* bufs[kPeerMax];        // every rank's gather buffer (peer pointers; own at [rank])
  unsigned* arrive[kPeerMax];     // every rank's arrival counters (peer pointers)
  unsigned* expected;             // this rank's expected counts [world], device memory
  const uint8_t* src;             // this rank's shard
  long long shard_bytes;          // multiple of 16
  int world, rank;
  unsigned* fault;
};

__device__ __forceinline__ void st_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kPeerThreads) peer_allgather_kernel(const __grid_constant__ PeerGatherArgs a) {
  const long long n16 = a.shard_bytes / 16;
  const long long off = static_cast<long long>(a.rank) * a.shard_bytes;
  const uint4* src = reinterpret_cast<const uint4*>(a.src);
  // 1. my shard -> slot `rank` of every rank's buffer
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
    for (int q = 0; q < a.world; ++q) reinterpret_cast<uint4*>(a.bufs[q] + off)[i] = v;
  }
  // 2. announce this CTA's part on every rank
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.world) st_release_sys_add(a.arrive[threadIdx.x] + a.rank, 1u);
  // 3. CTA 0 waits for every rank's parts of this call
  if (blockIdx.x == 0) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    if (threadIdx.x < a.world) {
      const unsigned want = a.expected[threadIdx.x] + gridDim.x;
      const unsigned* mine = a.arrive[a.rank] + threadIdx.x;
      const unsigned long long t0 = global_ns();
      // counters wrap after 2^32 parts; the signed difference stays valid
      while (static_cast<int>(ld_acquire_sys(mine) - want) < 0) {
        if (global_ns() - t0 > kWaitLimitNs) {
          failed = 1;
          break;
        }
      }
      a.expected[threadIdx.x] = want;
    }
    __syncthreads();
    if (threadIdx.x == 0 && failed) atomicOr(a.fault, kFaultFullWait);
  }
}

}  // namespace qlin
