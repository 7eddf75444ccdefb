// C ABI of the qlin library: argument validation, launch planning, TMA
// descriptor encoding and kernel launch.  Declarations: include/qlin.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "../../include/qlin.h"
#include "args.cuh"
#include "quant.cuh"
#include "peer.cuh"
#include "producers.cuh"
#include "decode.cuh"
#include "prefill_attn.cuh"
#include "prefill_delta.cuh"
#include "tcgemm.cuh"
#include "tcgemm_w4.cuh"
#include "tcgemv.cuh"
#include "dpgemv.cuh"

namespace qlin {

__device__ unsigned int g_qlin_fault;

// Scratch of qlin_peer_allgather_static, held by every GPU that loads this
// library until the process exits: the gather buffer, the arrival counter the
// kernel adds to and its expected count.  Device statics are zero when the
// module loads; the counters only ever grow.
constexpr size_t kStaticGatherBytes = QLIN_STATIC_GATHER_MAX_BYTES;
static __device__ __align__(256) uint8_t g_static_gather[kStaticGatherBytes];
static __device__ __align__(256) unsigned g_static_arrive[kPeerMax];
static __device__ __align__(256) unsigned g_static_expected[kPeerMax];

namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kMaxDevices = 64;

thread_local char g_err[512];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(QLIN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Every kernel of the library runs with the largest shared-memory carveout
// (once per kernel and device).  A CTA can only be placed on an SM whose
// L1 / shared-memory split suits it; left to the driver's per-kernel choice,
// a launch placed early under programmatic dependent launch can find the
// SMs held by its predecessor's CTAs at a smaller split and wait for them to
// drain.  One split for all keeps consecutive launches co-resident.
int prefer_shared(const void* kern) {
  static std::mutex mu;
  static std::unordered_map<const void*, unsigned long long> done;  // kernel -> devices configured
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return QLIN_OK;  // the launch itself reports the error
  }
  const unsigned long long bit = 1ull << (dev & 63);
  std::lock_guard<std::mutex> g(mu);
  unsigned long long& mask = done[kern];
  if (mask & bit) return QLIN_OK;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(carveout)");
  mask |= bit;
  return QLIN_OK;
}

// ---------------------------------------------------------------- device info
struct DevInfo {
  int dev = -1;
  int sms = 0;
  unsigned* fault = nullptr;                // device fault word of this GPU
  volatile unsigned* fault_host = nullptr;  // its host-visible mirror, or null
};

DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// One mapped pinned host word per device: the kernels' record_fault stores to
// it, so every later entry point sees a fault without synchronising.
unsigned* g_fault_host = nullptr;

int device_info_setup(int dev, bool mirror, DevInfo* out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DevInfo& d = g_dev[dev];
  cudaError_t e;
  if (d.sms == 0) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    void* fp = nullptr;
    e = cudaGetSymbolAddress(&fp, g_qlin_fault);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_qlin_fault)");
    d.fault = static_cast<unsigned*>(fp);
    d.dev = dev;
    d.sms = sms;
  }
  if (mirror && !d.fault_host) {
    if (!g_fault_host) {
      void* h = nullptr;
      e = cudaHostAlloc(&h, kMaxDevices * sizeof(unsigned), cudaHostAllocMapped | cudaHostAllocPortable);
      if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(fault mirror)");
      memset(h, 0, kMaxDevices * sizeof(unsigned));
      g_fault_host = static_cast<unsigned*>(h);
    }
    void* dp = nullptr;
    e = cudaHostGetDevicePointer(&dp, g_fault_host + dev, 0);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostGetDevicePointer(fault mirror)");
    e = cudaMemcpyToSymbol(g_qlin_fault_host, &dp, sizeof(dp));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(fault mirror)");
    d.fault_host = g_fault_host + dev;
  }
  *out = d;
  return QLIN_OK;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(QLIN_ERR_UNSUPPORTED, "device index %d", *dev);
  return QLIN_OK;
}

// Device attributes, fault word and fault mirror of the current device.  The
// first call on a device sets them up (and allocates the pinned mirror once
// per process).
int device_info(DevInfo* out) {
  int dev = 0;
  if (int r = current_device(&dev)) return r;
  const DevInfo& d = g_dev[dev];
  if (d.sms != 0 && d.fault_host) {
    *out = d;
    return QLIN_OK;
  }
  return device_info_setup(dev, true, out);
}

// As device_info, without the host mirror: allocates nothing.
int device_info_noalloc(DevInfo* out) {
  int dev = 0;
  if (int r = current_device(&dev)) return r;
  const DevInfo& d = g_dev[dev];
  if (d.sms != 0) {
    *out = d;
    return QLIN_OK;
  }
  return device_info_setup(dev, false, out);
}

// Entry points report a fault recorded by an earlier launch on this device
// (a bounded device wait that gave up) until qlin_device_fault(1) clears it.
int sticky_fault(const DevInfo& d) {
  if (d.fault_host && *d.fault_host)
    return fail(QLIN_ERR_DEVICE_FAULT,
                "a bounded device-side wait of an earlier launch on device %d gave up; its results are "
                "invalid (read and clear with qlin_device_fault(1))",
                d.dev);
  return QLIN_OK;
}

// device_info + sticky_fault: what every launching entry point calls first.
int launch_info(DevInfo* out) {
  if (int r = device_info(out)) return r;
  return sticky_fault(*out);
}

// ---------------------------------------------------------------- TMA descriptors
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int encode_fn(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::call_once(g_encode_once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!g_encode) return fail(QLIN_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  *fn = g_encode;
  return QLIN_OK;
}

// cuMemGetAddressRange through the runtime's driver entry point (the base of
// the allocation that holds a pointer, for CUDA IPC offsets).
typedef CUresult (*PfnAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);
std::once_flag g_range_once;
PfnAddressRange g_range = nullptr;
int address_range(const void* p, CUdeviceptr* base) {
  std::call_once(g_range_once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PfnAddressRange>(f);
  });
  if (!g_range) return fail(QLIN_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
  size_t size = 0;
  if (g_range(base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "pointer is not a device allocation");
  return QLIN_OK;
}

// Row-major 2-D tensor [rows, cols] with `row_bytes` between rows, loaded in
// boxes of [box_rows, box_cols].
// Encoded tensor maps are cached by every encode parameter (a map describes
// an address range and a layout, never the contents), so the weights and the
// engine's reused workspace buffers are encoded once.  The cache is a hash
// table (a layer's launches look up several maps each, among hundreds of
// weights); when it reaches kMapCache entries it starts over.
struct MapKey {
  const void* base;
  uint64_t cols, rows, row_bytes;
  uint32_t box_cols, box_rows, dt, sw;
  bool operator==(const MapKey& o) const {
    return base == o.base && cols == o.cols && rows == o.rows && row_bytes == o.row_bytes &&
           box_cols == o.box_cols && box_rows == o.box_rows && dt == o.dt && sw == o.sw;
  }
};
inline uint64_t mix64(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
  return h;
}
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = reinterpret_cast<uintptr_t>(k.base);
    h = mix64(h, k.cols);
    h = mix64(h, k.rows);
    h = mix64(h, k.row_bytes);
    h = mix64(h, (static_cast<uint64_t>(k.box_cols) << 32) | k.box_rows);
    h = mix64(h, (static_cast<uint64_t>(k.dt) << 32) | k.sw);
    return static_cast<size_t>(h);
  }
};
constexpr size_t kMapCache = 8192;
struct MapCache {
  std::mutex mu;
  std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
};
MapCache& map_cache() {
  static MapCache c;
  return c;
}

int encode_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
               uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, bool sw128);

int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
             uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, bool sw128 = false) {
  const MapKey k{base, cols, rows, row_bytes, box_cols, box_rows, static_cast<uint32_t>(dt), sw128 ? 1u : 0u};
  MapCache& c = map_cache();
  {
    std::lock_guard<std::mutex> g(c.mu);
    auto it = c.maps.find(k);
    if (it != c.maps.end()) {
      *m = it->second;
      return QLIN_OK;
    }
  }
  if (int r = encode_map(m, base, dt, cols, rows, row_bytes, box_cols, box_rows, sw128)) return r;
  std::lock_guard<std::mutex> g(c.mu);
  if (c.maps.size() >= kMapCache) c.maps.clear();
  c.maps.emplace(k, *m);
  return QLIN_OK;
}

int encode_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
               uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, bool sw128) {
  PFN_cuTensorMapEncodeTiled_v12000 fn;
  if (int r = encode_fn(&fn)) return r;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {row_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QLIN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) cols=%llu rows=%llu", (int)r,
                (unsigned long long)cols, (unsigned long long)rows);
  return QLIN_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Planner constants.  A build with -DQLIN_TUNING reads overrides of them
// from the environment once (for on-box sweeps); the shipped library has no
// run-time switches.  They change scheduling and the fp32 summation order of
// the K split only, never the integer results.
//   split          K split / cluster size (0: planner's choice)
//   budget_kb      per-CTA shared-memory budget (0: 112 KB, 200 KB at one CTA per SM)
//   ctas_per_sm    cap on co-resident CTAs per SM (0: from tensor memory)
//   max_level      highest batch-plan level tried (2: one batch)
//   stream_kb      shared-memory budget of long streamed launches (0: planner's)
//   max_cluster    largest K split considered
//   rb_max         weight-ring slots of a streamed plan (0: 3 short, 4 long launches)
//   half           128-column halves per prefill tile for plain outputs (0/1: 1; 2: two)
//   prefill_min_m  rows from which projections take the tensor-core GEMM
//   pdl            programmatic dependent launch (1: on)
#ifdef QLIN_TUNING
int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  return (e && *e) ? atoi(e) : dflt;
}
#define QLIN_KNOB(fn, env, dflt) \
  int fn() {                     \
    static const int v = env_int(env, dflt); \
    return v;                    \
  }
#else
#define QLIN_KNOB(fn, env, dflt) \
  constexpr int fn() { return dflt; }
#endif
QLIN_KNOB(tune_split, "QLIN_TUNE_SPLIT", 0)
QLIN_KNOB(tune_pdl, "QLIN_TUNE_PDL", 1)
QLIN_KNOB(tune_budget, "QLIN_TUNE_BUDGET_KB", 0)
QLIN_KNOB(tune_ctas_per_sm, "QLIN_TUNE_CTAS_PER_SM", 0)
QLIN_KNOB(tune_max_level, "QLIN_TUNE_MAX_LEVEL", 2)
QLIN_KNOB(tune_stream_budget, "QLIN_TUNE_STREAM_BUDGET_KB", 0)
QLIN_KNOB(tune_max_cluster, "QLIN_TUNE_MAX_CLUSTER", 8)
QLIN_KNOB(tune_rb_max, "QLIN_TUNE_RB_MAX", 0)
QLIN_KNOB(tune_half, "QLIN_TUNE_HALF", 0)
QLIN_KNOB(prefill_min_m, "QLIN_PREFILL_MIN_M", 128)
QLIN_KNOB(tune_timeline, "QLIN_TIMELINE", 0)
QLIN_KNOB(tune_dp, "QLIN_TUNE_DP", 1)  // 0: decode rows take the tensor-core kernel
// dp kernel weight ring: 0 never, 1 when resident weights need more than one
// wave, 2 whenever a ring plan exists
QLIN_KNOB(tune_dp_stream, "QLIN_TUNE_DP_STREAM", 1)
QLIN_KNOB(tune_dp_maxm, "QLIN_TUNE_DP_MAXM", 4)  // rows the dp kernel may serve
QLIN_KNOB(tune_ad_smax, "QLIN_TUNE_AD_SMAX", 8)  // attn_decode: largest cluster
QLIN_KNOB(tune_dp_m4, "QLIN_TUNE_DP_M4", 0)  // 1: 3-4 rows take any dp plan (W8 too)
QLIN_KNOB(tune_dp_m4ring, "QLIN_TUNE_DP_M4RING", 1)  // 0: 3-4 rows never take a ring plan
QLIN_KNOB(tune_ad_hsplit, "QLIN_TUNE_AD_HSPLIT", 0)  // attn_decode: forced query-head split (0: planner)
QLIN_KNOB(tune_kparts, "QLIN_TUNE_KPARTS", 0)  // W4 GEMM: forced K parts per tile (0: planner)
#undef QLIN_KNOB

bool use_dp() { return tune_dp() != 0; }

// Timeline slot of the next small-M launch: tuning builds with
// QLIN_TIMELINE=1 stamp each launch's phases into slot (launch count % 16).
int tl_next_slot() {
#ifdef QLIN_TUNING
  static std::atomic<int> next{0};
  if (tune_timeline()) return next.fetch_add(1) % kTlSlots;
#endif
  return -1;
}

// ---------------------------------------------------------------- tcgen05 path planning / launch
// Activation rows per row block: 1..16, and 32 for W8 (the W4 drain of 32
// rows does not fit its register budget).
int tc_mr(int wb, int64_t M) {
  const int mr = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : M <= 16 ? 16 : 32;
  return (wb == 4 && mr > 16) ? 16 : mr;
}

// Largest K split (thread-block cluster size, the portable maximum).
constexpr int kMaxCluster = 8;
// Dynamic shared memory one CTA may use (B200: 227 KB).
constexpr size_t kTcMaxSmem = 227 * 1024;

struct TcPlan {
  int split, gmax, bs, rb, ab, nbb, alias;
  // 2: one batch (weights in flight and operands complete before the grid
  // dependency); 0: weights stream through double-buffered batches.
  int level;
  size_t smem;
};

// Batch plan for one K split, first that fits the per-CTA budget of
// ~112 KB (two CTAs per SM) and the 256-column tensor-memory share:
//  1. one batch: the whole K range in flight, one hand-off per role (tried
//     without, then with, the partial-sum buffer aliased onto rank 0's
//     finished operand region);
//  2. double-buffered batches (the weights stream behind the MMAs).
// (A plan with every packed W4 group resident and a ring of unpacked tiles
// was measured slower than streaming once the W4 operands became the masked
// nibble tiles: 12.3 vs 10.8 us for the config-2 gate/up at split 4.)
void plan_batches(int wb, int mr, int ns, int wgrp, long long ctas, int sms, bool long_stream, bool one_per_sm,
                  TcPlan& pl) {
  // A kernel instance whose registers fit only one CTA per SM (the 8- to
  // 32-row blocks) shares no SM with the next launch anyway: it may use most
  // of shared memory.  Measured on B200, config-2 shapes at M = 16: fused
  // gate/up 29.4 -> 20.0 us, down 22.4 -> 11.0 us.
  const uint32_t budget = (tune_budget() > 0 ? tune_budget() : one_per_sm ? 200 : 112) * 1024;
  // A long streamed launch (tens of MB of weights) that fits one CTA per SM
  // may use most of shared memory for a deeper weight ring; its weight
  // stream, not the next launch's prologue, is what bounds it.
  const uint32_t stream_budget =
      tune_stream_budget() > 0 ? tune_stream_budget() * 1024u
                               : ((long_stream && ctas <= sms) || one_per_sm ? 200u * 1024 : budget);
  const int s = pl.split, gmax = pl.gmax;
  const TcLayout base = tc_layout(wb, mr, ns, wgrp, gmax, 1, 1, 1, 1, s, 0);
  const int tmem_groups = static_cast<int>(kTmemBudget / base.per_buf);
  auto fits = [&](int bs, int rb, int ab, int nbb, int alias) {
    const TcLayout L = tc_layout(wb, mr, ns, wgrp, gmax, bs, rb, ab, nbb, s, alias);
    if (alias && (s < 2 || L.part_bytes > L.op_bytes)) return false;
    if (L.total > budget) return false;
    pl.bs = bs;
    pl.rb = rb;
    pl.ab = ab;
    pl.nbb = nbb;
    pl.alias = alias;
    return true;
  };
  bool ok = false;
  pl.level = 0;
  for (int alias = 0; alias < 2 && !ok && tune_max_level() >= 2; ++alias)
    if (gmax <= tmem_groups && fits(gmax, 1, wb == 4 ? 1 : 0, 1, alias)) ok = true, pl.level = 2;
  if (!ok) {
    // Streamed: the most groups in flight (weight-ring slots x groups per
    // batch) that fit, preferring larger batches (fewer hand-offs).
    const int ab = wb == 4 ? 2 : 0;
    int best_bs = 1, best_rb = 2;
    // (three slots for short launches: measured on the config-2 shapes, the
    // fused gate/up takes 9.9 us with three, 10.6 us with two)
    const int rb_max = tune_rb_max() > 0 ? tune_rb_max() : long_stream ? 4 : 3;
    for (int rb = 2; rb <= rb_max; ++rb) {
      const TcLayout one = tc_layout(wb, mr, ns, wgrp, gmax, 1, rb, ab, 2, s, 0);
      const uint32_t per_group = rb * base.raw_stage + (wb == 4 ? ab * ns * base.atile : 0);
      const uint32_t fixed = one.total - per_group;
      const uint32_t room = stream_budget > fixed ? stream_budget - fixed : 0;
      int bs = static_cast<int>(room / per_group);
      if (bs > tmem_groups / 2) bs = tmem_groups / 2;
      if (bs > (gmax + rb - 1) / rb) bs = (gmax + rb - 1) / rb;
      if (bs < 1) continue;
      if (rb * bs > best_rb * best_bs || (rb * bs == best_rb * best_bs && bs > best_bs)) {
        best_bs = bs;
        best_rb = rb;
      }
    }
    pl.bs = best_bs;
    pl.rb = best_rb;
    pl.ab = ab;
    pl.nbb = 2;
    pl.alias = 0;
  }
  const TcLayout L = tc_layout(wb, mr, ns, wgrp, gmax, pl.bs, pl.rb, pl.ab, pl.nbb, s, pl.alias);
  // At most 512 / tmem_cols CTAs may share an SM, or a tensor-memory
  // allocation could wait on a CTA of the next launch: pad shared memory so
  // that no more CTAs than that fit.
  uint32_t max_ctas = 512 / L.tmem_cols;
  if (tune_ctas_per_sm() > 0 && static_cast<uint32_t>(tune_ctas_per_sm()) < max_ctas) max_ctas = tune_ctas_per_sm();
  uint32_t smem = L.total;
  const uint32_t floor_smem = (228 * 1024) / (max_ctas + 1) - 1024 + 16;
  if (smem < floor_smem) smem = floor_smem;
  pl.smem = smem;
}

// Choose the K split (cluster size).  Per launch the critical path after
// the grid dependency is activation load -> MMA -> drain -> cluster combine,
// and the combine grows with the split; the weight stream itself overlaps the
// preceding kernel.  Measured on B200 (config-2 layer shapes, K = 2048..6144)
// the best split is the largest one (up to 8) that keeps the launch at about
// 1.3 CTAs per SM: more CTAs leave clusters waiting for the previous
// launch's CTAs to retire, fewer leave HBM under-subscribed.
int active_clusters(int wb, int mr, int ns, int split, size_t smem);
int blocks_by_regs(int wb, int mr, int ns);

// Clusters of `s` CTAs that stay resident at once for a plan with `smem`
// bytes and `tmem_cols` tensor-memory columns per CTA, or -1 without a
// device.  A cluster must fit one GPC, so the count depends on the GPCs'
// sizes, not only on the SM count: on B200, clusters of 7 CTAs at one CTA
// per SM place only 15 at once (105 CTAs), clusters of 6 place 22.
// cudaOccupancyMaxActiveClusters counts one CTA per SM; with two per SM a
// GPC of g SMs offers 2g slots, so a cluster of s places like one of s/2
// (the mean of the two neighbours for odd s).
long long cluster_capacity(int wb, int mr, int ns, int s, size_t smem, uint32_t tmem_cols) {
  long long per_sm = (228 * 1024) / (static_cast<long long>(smem) + 1024);
  const long long by_tmem = tmem_cols ? 512 / tmem_cols : 1;
  if (by_tmem < per_sm) per_sm = by_tmem;
  const long long by_regs = blocks_by_regs(wb, mr, ns);
  if (by_regs > 0 && by_regs < per_sm) per_sm = by_regs;
  auto c1 = [&](int x) { return static_cast<long long>(active_clusters(wb, mr, ns, x, smem)); };
  if (per_sm <= 1) return c1(s);
  if (s == 1) {
    const long long a = c1(1);
    return a < 0 ? -1 : 2 * a;
  }
  if (s % 2 == 0) return c1(s / 2);
  const long long a = c1((s - 1) / 2), b = c1((s + 1) / 2);
  return (a < 0 || b < 0) ? -1 : (a + b) / 2;
}

TcPlan plan_tc(int wb, int mr, int ns, int K, int wgrp, int tiles, int rowblocks, int sms, bool query) {
  const int G = K / kGroup;
  // CTAs per SM that the instance's registers allow (from the device when it
  // is queried): with one, the targets below count one CTA per SM.
  const int reg_blocks = query ? blocks_by_regs(wb, mr, ns) : -1;
  const bool one_per_sm = reg_blocks == 1;
  const long long target = one_per_sm ? sms : (static_cast<long long>(sms) * 4 + 2) / 3;  // ~1.33 CTAs per SM
  const long long two_per_sm = one_per_sm ? sms : 2ll * sms;
  // Per plan level: the largest split within the CTA target, and the
  // smallest split beyond it (within two CTAs per SM).
  TcPlan in[3] = {}, up[3] = {}, any{}, stream{}, compact{};
  long long stream_inflight = -1;
  // Weight bytes of the launch: past ~16 MB (the config-2 launches are at
  // most 13 MB) the launch is a long HBM stream rather than a short step
  // between two dependencies.
  const long long wbytes = static_cast<long long>(tiles) * ns * kTileN * K / (wb == 8 ? 1 : 2);
  const bool long_stream = wbytes >= (16ll << 20);
  const int cmax = tune_max_cluster() < kMaxCluster ? tune_max_cluster() : kMaxCluster;
  const int smax = G < cmax ? G : cmax;
  for (int s = 1; s <= smax; ++s) {
    TcPlan pl{s, (G + s - 1) / s, 1, 1, 0, 1, 0, 0, 0};
    if (tune_split() > 0 && s != tune_split() && tune_split() <= smax) continue;  // (tuning builds only)
    const long long ctas = static_cast<long long>(tiles) * s * rowblocks;
    plan_batches(wb, mr, ns, wgrp, ctas, sms, long_stream, one_per_sm, pl);
    if (pl.smem > kTcMaxSmem) continue;
    if (tune_split() == s) return pl;
    if (any.split == 0) any = pl;  // smallest feasible split, whatever its size
    const TcLayout L = tc_layout(wb, mr, ns, wgrp, pl.gmax, pl.bs, pl.rb, pl.ab, pl.nbb, s, pl.alias);
    // Resident clusters (from the device's GPC layout when it is queried)
    // and whether the launch's clusters fit in one wave.
    const long long clusters = static_cast<long long>(tiles) * rowblocks;
    const long long cap = query ? cluster_capacity(wb, mr, ns, s, pl.smem, L.tmem_cols) : -1;
    const bool one_wave = cap < 0 || clusters <= cap;
    if (pl.level == 0 && long_stream) {
      // Long streamed launches are bound by the weight bytes in flight over
      // the whole GPU: resident CTAs x ring slots x groups per batch, divided
      // by the waves the launch needs (measured on the config-5 shapes).
      long long per_sm = (228 * 1024) / (static_cast<long long>(pl.smem) + 1024);
      if (one_per_sm) per_sm = 1;
      const long long slots = cap > 0 ? cap * s : sms * (per_sm < 1 ? 1 : per_sm);
      const long long resident = ctas < slots ? ctas : slots;
      const long long waves = (ctas + slots - 1) / slots;  // a second wave serialises behind the first
      const long long inflight = resident * pl.rb * pl.bs * L.raw_stage / waves;
      if (inflight > stream_inflight) {
        stream_inflight = inflight;
        stream = pl;
      }
      continue;
    }
    // One-batch plans with at most one CTA per SM, at most 8 groups per CTA
    // and clusters of at most 6 (the largest such split).
    if (pl.level == 2 && ctas <= sms && pl.gmax <= 8 && s <= 6 && one_wave) compact = pl;
    const bool within = ctas <= target && one_wave;
    if (within || (s == 1 && in[pl.level].split == 0)) in[pl.level] = pl;
    else if (ctas <= two_per_sm && one_wave && up[pl.level].split == 0) up[pl.level] = pl;
  }
  if (long_stream) in[0] = stream, up[0] = TcPlan{};
  // A compact one-batch plan first.  Measured on B200 (config-2 shapes): the
  // o projection (16 tiles, K = 2048) takes 4.1 us at split 6 (96 CTAs) and
  // 4.6 us at split 8; the qkv projection (32 tiles) 5.1 us at split 4 (128
  // CTAs) and 5.6 us at split 6 (192 CTAs).  Where none exists (the W8
  // config-1 GEMV needs 11 groups per CTA at split 3, and is fastest at split
  // 4 with 192 CTAs), the CTA-target rule below applies.
  if (compact.split) return compact;
  // Within the CTA target, the highest level first (more of the work ahead
  // of the grid dependency); only then beyond the target, where extra splits
  // add combine work, the smallest one.  Measured on B200 with the W4
  // nibble-split operands: the one-batch plan of the fused gate/up needs
  // split 6 (288 CTAs) to fit and takes 15.5 us, the streamed plan at split 4
  // (192 CTAs) 10.8 us.
  for (int lv = 2; lv >= 0; --lv)
    if (in[lv].split) return in[lv];
  for (int lv = 2; lv >= 0; --lv)
    if (up[lv].split) return up[lv];
  return any;
}

// Opt the kernel instance in to the full dynamic shared memory (once per device).
template <int WB, int MR, int EPI>
int configure_tc() {
  auto kern = tc_gemv_kernel<WB, MR, EPI>;
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
    if (int r = prefer_shared(reinterpret_cast<const void*>(kern))) return r;
    configured.fetch_or(bit);
  }
  return QLIN_OK;
}

// Clusters of `split` CTAs with `smem` bytes each that the device keeps
// resident at once (cudaOccupancyMaxActiveClusters: it accounts for the
// GPC a cluster must fit in, registers and shared memory), or -1.
template <int WB, int MR, int EPI>
int active_clusters_t(int split, size_t smem) {
  if (configure_tc<WB, MR, EPI>() != QLIN_OK) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(split, 1, 1);
  cfg.blockDim = dim3(tc_threads(WB), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_gemv_kernel<WB, MR, EPI>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return n;
}

template <int WB, int EPI>
int active_clusters_mr(int mr, int split, size_t smem) {
  switch (mr) {
    case 1: return active_clusters_t<WB, 1, EPI>(split, smem);
    case 2: return active_clusters_t<WB, 2, EPI>(split, smem);
    case 4: return active_clusters_t<WB, 4, EPI>(split, smem);
    case 8: return active_clusters_t<WB, 8, EPI>(split, smem);
    case 16: return active_clusters_t<WB, 16, EPI>(split, smem);
    default:
      if constexpr (WB == 8) return active_clusters_t<WB, 32, EPI>(split, smem);
      return -1;
  }
}

struct ClusterKey {
  int dev, wb, mr, ns, split;
  size_t smem;
  bool operator==(const ClusterKey& o) const {
    return dev == o.dev && wb == o.wb && mr == o.mr && ns == o.ns && split == o.split && smem == o.smem;
  }
};
struct ClusterKeyHash {
  size_t operator()(const ClusterKey& k) const {
    uint64_t h = mix64(static_cast<uint64_t>(k.smem), (static_cast<uint64_t>(k.dev) << 32) | k.split);
    return static_cast<size_t>(mix64(h, (static_cast<uint64_t>(k.wb) << 16) | (k.mr << 4) | k.ns));
  }
};

// Resident-cluster capacity of the small-M kernel for a plan (cached), or -1
// when no device answers (the planner then counts shared-memory slots).
int active_clusters(int wb, int mr, int ns, int split, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<ClusterKey, int, ClusterKeyHash> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  const ClusterKey k{dev, wb, mr, ns, split, smem};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(k);
    if (it != cache.end()) return it->second;
  }
  int n;
  if (wb == 8) n = ns == 1 ? active_clusters_mr<8, kEpiOut>(mr, split, smem) : active_clusters_mr<8, kEpiSiluQuant>(mr, split, smem);
  else n = ns == 1 ? active_clusters_mr<4, kEpiOut>(mr, split, smem) : active_clusters_mr<4, kEpiSiluQuant>(mr, split, smem);
  std::lock_guard<std::mutex> g(mu);
  cache.emplace(k, n);
  return n;
}

// CTAs of a kernel instance that share one SM by registers: two when the
// instance's registers x threads fit half of the 64K-register file, else
// one, or -1.  (This matches what runs: per-CTA timelines show two CTAs per
// SM for the 1- to 4-row instances, 78-98 registers; the 8- to 32-row
// instances use 112-200.  cudaOccupancyMaxActiveBlocksPerMultiprocessor
// answers one for all of them, so it is not used.)
template <int WB, int MR, int EPI>
int blocks_by_regs_t() {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, tc_gemv_kernel<WB, MR, EPI>) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return static_cast<long long>(fa.numRegs) * tc_threads(WB) * 2 <= 65536 ? 2 : 1;
}

template <int WB, int EPI>
int blocks_by_regs_mr(int mr) {
  switch (mr) {
    case 1: return blocks_by_regs_t<WB, 1, EPI>();
    case 2: return blocks_by_regs_t<WB, 2, EPI>();
    case 4: return blocks_by_regs_t<WB, 4, EPI>();
    case 8: return blocks_by_regs_t<WB, 8, EPI>();
    case 16: return blocks_by_regs_t<WB, 16, EPI>();
    default:
      if constexpr (WB == 8) return blocks_by_regs_t<WB, 32, EPI>();
      return -1;
  }
}

// Per device, kernel family and row block (cached).  W8 gate/up has two
// epilogues; the smaller count of the two is used.
int blocks_by_regs(int wb, int mr, int ns) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  const uint64_t k = (static_cast<uint64_t>(dev) << 32) | (static_cast<uint64_t>(wb) << 16) | (mr << 4) | ns;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(k);
    if (it != cache.end()) return it->second;
  }
  int n;
  if (wb == 8) {
    if (ns == 1) {
      n = blocks_by_regs_mr<8, kEpiOut>(mr);
    } else {
      const int a = blocks_by_regs_mr<8, kEpiSiluBf16>(mr), b = blocks_by_regs_mr<8, kEpiSiluQuant>(mr);
      n = (a < 0 || b < 0) ? -1 : (a < b ? a : b);
    }
  } else {
    n = ns == 1 ? blocks_by_regs_mr<4, kEpiOut>(mr) : blocks_by_regs_mr<4, kEpiSiluQuant>(mr);
  }
  std::lock_guard<std::mutex> g(mu);
  cache.emplace(k, n);
  return n;
}

template <int WB, int MR, int EPI>
int launch_tc_t(const GemvArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = tc_gemv_kernel<WB, MR, EPI>;
  if (int r = configure_tc<WB, MR, EPI>()) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(tc_threads(WB), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = grid.x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = tune_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(tc_gemv)");
  return QLIN_OK;
}

template <int WB, int EPI>
int launch_tc_mr(int mr, const GemvArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
  switch (mr) {
    case 1: return launch_tc_t<WB, 1, EPI>(a, grid, smem, st);
    case 2: return launch_tc_t<WB, 2, EPI>(a, grid, smem, st);
    case 4: return launch_tc_t<WB, 4, EPI>(a, grid, smem, st);
    case 8: return launch_tc_t<WB, 8, EPI>(a, grid, smem, st);
    case 16: return launch_tc_t<WB, 16, EPI>(a, grid, smem, st);
    default:
      if constexpr (WB == 8) return launch_tc_t<WB, 32, EPI>(a, grid, smem, st);
      return fail(QLIN_ERR_UNSUPPORTED, "row block %d", mr);
  }
}

// Row block and K split for the tcgen05 path.  Row blocks of 32 rows hold
// the largest activation and partial-sum buffers; when no split of K fits
// shared memory, 16-row blocks are used.  Returns QLIN_OK or an error.
int choose_tc_uncached(int wb, int ns, int64_t M, int K, int wgrp, int tiles, int sms, bool query, int* mr_out,
                       int* rowblocks_out, TcPlan* pl_out) {
  int mr = tc_mr(wb, M);
  for (;;) {
    const int nm = mr < 16 ? 16 : mr;
    const int64_t rowblocks = (M + nm - 1) / nm;
    if (rowblocks > 65535 || tiles > 65535) return fail(QLIN_ERR_SHAPE, "grid too large (M=%lld)", (long long)M);
    const TcPlan pl = plan_tc(wb, mr, ns, K, wgrp, tiles, static_cast<int>(rowblocks), sms, query);
    if (pl.split > 0) {
      *mr_out = mr;
      *rowblocks_out = static_cast<int>(rowblocks);
      *pl_out = pl;
      return QLIN_OK;
    }
    if (mr <= 16) break;
    mr = 16;
  }
  return fail(QLIN_ERR_SHAPE, "K=%d exceeds the shared-memory capacity of the small-M kernel", K);
}

// The plan depends only on these inputs (the tuning overrides are read once
// per process), so it is computed once per shape and looked up afterwards.
struct TcKey {
  int wb, ns, K, wgrp, tiles, sms, dev;  // dev = -1: planned without querying a device
  int64_t M;
  bool operator==(const TcKey& o) const {
    return wb == o.wb && ns == o.ns && K == o.K && wgrp == o.wgrp && tiles == o.tiles && sms == o.sms &&
           dev == o.dev && M == o.M;
  }
};
struct TcKeyHash {
  size_t operator()(const TcKey& k) const {
    uint64_t h = static_cast<uint64_t>(k.M);
    h = mix64(h, (static_cast<uint64_t>(k.wb) << 40) ^ (static_cast<uint64_t>(k.ns) << 32) ^ static_cast<uint32_t>(k.K));
    h = mix64(h, (static_cast<uint64_t>(static_cast<uint32_t>(k.wgrp)) << 32) ^ static_cast<uint32_t>(k.tiles));
    h = mix64(h, static_cast<uint64_t>(static_cast<uint32_t>(k.dev)));
    return static_cast<size_t>(mix64(h, static_cast<uint64_t>(k.sms)));
  }
};
struct TcChoice {
  int mr, rowblocks;
  TcPlan pl;
};
constexpr size_t kPlanCache = 4096;
struct PlanCache {
  std::mutex mu;
  std::unordered_map<TcKey, TcChoice, TcKeyHash> plans;
};
PlanCache& plan_cache() {
  static PlanCache c;
  return c;
}

// `query`: plan with the current device's cluster capacity (launch path);
// without it (the CPU plan query) clusters are counted by shared-memory slots.
int choose_tc(int wb, int ns, int64_t M, int K, int wgrp, int tiles, int sms, bool query, int* mr_out,
              int* rowblocks_out, TcPlan* pl_out) {
  int dev = -1;
  if (query && cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
    query = false;
  }
  const TcKey k{wb, ns, K, wgrp, tiles, sms, dev, M};
  PlanCache& c = plan_cache();
  {
    std::lock_guard<std::mutex> g(c.mu);
    auto it = c.plans.find(k);
    if (it != c.plans.end()) {
      *mr_out = it->second.mr;
      *rowblocks_out = it->second.rowblocks;
      *pl_out = it->second.pl;
      return QLIN_OK;
    }
  }
  TcChoice ch{};
  if (int r = choose_tc_uncached(wb, ns, M, K, wgrp, tiles, sms, query, &ch.mr, &ch.rowblocks, &ch.pl)) return r;
  {
    std::lock_guard<std::mutex> g(c.mu);
    if (c.plans.size() >= kPlanCache) c.plans.clear();
    c.plans.emplace(k, ch);
  }
  *mr_out = ch.mr;
  *rowblocks_out = ch.rowblocks;
  *pl_out = ch.pl;
  return QLIN_OK;
}

int run_tc(int wb, int epi, GemvArgs& a, int tiles, cudaStream_t st) {
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  const int ns = epi == kEpiOut ? 1 : 2;
  int mr = 0, rowblocks = 0;
  TcPlan pl{};
  if (int r = choose_tc(wb, ns, a.M, a.K, a.wgrp, tiles, di.sms, true, &mr, &rowblocks, &pl)) return r;
  const int nm = mr < 16 ? 16 : mr;
  if (int r = make_map(&a.ta, a.a_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.K, a.M, a.K, 128, nm, true)) return r;
  a.split = pl.split;
  a.gmax = pl.gmax;
  a.bs = pl.bs;
  a.rb = pl.rb;
  a.ab = pl.ab;
  a.nbb = pl.nbb;
  a.part_alias = pl.alias;
  a.fault = di.fault;
  a.tl_slot = tl_next_slot();
  const dim3 grid(pl.split, tiles, rowblocks);
  if (wb == 8) {
    switch (epi) {
      case kEpiOut: return launch_tc_mr<8, kEpiOut>(mr, a, grid, pl.smem, st);
      case kEpiSiluBf16: return launch_tc_mr<8, kEpiSiluBf16>(mr, a, grid, pl.smem, st);
      default: return launch_tc_mr<8, kEpiSiluQuant>(mr, a, grid, pl.smem, st);
    }
  }
  switch (epi) {
    case kEpiOut: return launch_tc_mr<4, kEpiOut>(mr, a, grid, pl.smem, st);
    default: return launch_tc_mr<4, kEpiSiluQuant>(mr, a, grid, pl.smem, st);
  }
}

// ---------------------------------------------------------------- tensor-core GEMM (large M)
template <int EPI, int HS = 2>
int launch_prefill_w8(const GemmArgs& g, int grid, cudaStream_t st) {
  auto kern = tc_gemm_kernel<EPI, HS>;
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGmSmem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc_gemm smem)");
    if (int r = prefer_shared(reinterpret_cast<const void*>(kern))) return r;
    configured.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kGmThreads, 1, 1);
  cfg.dynamicSmemBytes = kGmSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = tune_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(tc_gemm)");
  return QLIN_OK;
}

// epi: kEpiOut (gemm / proj3 segments) or the fused gate/up epilogues, whose
// two segments are gate and up with the same N.
int run_prefill_w8(int epi, const GemvArgs& a, int half_tiles, cudaStream_t st) {
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  GemmArgs g;
  memset(&g, 0, sizeof(g));
  if (int r = make_map(&g.ta, a.a_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.K, a.M, a.K, 128, kGmRows, true)) return r;
  bool vec = aligned(a.out, 16) && a.ldo % 8 == 0 && (!a.res || (aligned(a.res, 16) && a.ldr % 8 == 0));
  for (int i = 0; i < a.nseg; ++i) {
    g.seg[i] = a.seg[i];
    if (int r = make_map(&g.seg[i].tw, a.seg[i].w, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.seg[i].n, a.K, a.seg[i].n,
                         kTileN, 128, true))
      return r;
    vec = vec && a.seg[i].out_col % 8 == 0;
  }
  g.nseg = a.nseg;
  g.half_tiles = half_tiles;
  g.a_s = a.a_s;
  g.M = a.M;
  g.K = a.K;
  g.out = a.out;
  g.ldo = a.ldo;
  g.res = a.res;
  g.ldr = a.ldr;
  g.vec_out = vec ? 1 : 0;
  g.out_q = a.out_q;
  g.out_s = a.out_s;
  g.n_q = a.n_q;
  g.fault = di.fault;
  if (epi != kEpiOut) g.half_tiles = 2 * half_tiles;  // (gate tile, up tile) pairs
  const long long mtiles = (a.M + kGmRows - 1) / kGmRows;
  // Plain outputs take one 128-column half per tile (twice the tiles; a
  // separate kernel instance that drains half the columns per group and
  // spills nothing).  The fused gate/up keeps its (gate, up) tile pairs.
  // Measured on B200, config 3 (K = 2048, N = 12288): M = 2048 188 -> 157 us,
  // M = 512 67 -> 47 us; W8 K = 5120, N = 17408 at M = 64 67 -> 34 us.
  int hs = epi == kEpiOut ? 1 : 2;
#ifdef QLIN_TUNING
  if (epi == kEpiOut && tune_half() == 2) hs = 2;
#endif
  const long long tiles = mtiles * ((g.half_tiles + hs - 1) / hs);
  const int grid = static_cast<int>(tiles < di.sms ? tiles : di.sms);
  switch (epi) {
    case kEpiOut:
#ifdef QLIN_TUNING
      if (hs == 2) return launch_prefill_w8<kEpiOut>(g, grid, st);
#endif
      return launch_prefill_w8<kEpiOut, 1>(g, grid, st);
    case kEpiSiluBf16: return launch_prefill_w8<kEpiSiluBf16>(g, grid, st);
    default: return launch_prefill_w8<kEpiSiluQuant>(g, grid, st);
  }
}

template <int EPI, int HS = 2>
int launch_prefill_w4(const GemmW4Args& g, int grid, cudaStream_t st) {
  auto kern = tc_gemm_w4_kernel<EPI, HS>;
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kG4Smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc_gemm_w4 smem)");
    if (int r = prefer_shared(reinterpret_cast<const void*>(kern))) return r;
    configured.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kG4Threads, 1, 1);
  cfg.dynamicSmemBytes = kG4Smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = tune_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(tc_gemm_w4)");
  return QLIN_OK;
}

// Stream-ordered pool of the W4 GEMM's K-part workspaces, one per device,
// owned by the library.  Freed blocks stay in the pool (no release
// threshold), so an eager launch reuses the previous launch's memory instead
// of mapping new pages (a default pool trims at every synchronisation).
cudaMemPool_t g_ws_pool[kMaxDevices] = {};
std::mutex g_ws_pool_mu;

int ws_pool(int dev, cudaMemPool_t* pool) {
  if (dev < 0 || dev >= kMaxDevices) return fail(QLIN_ERR_CUDA, "device %d out of range", dev);
  std::lock_guard<std::mutex> g(g_ws_pool_mu);
  if (!g_ws_pool[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    cudaError_t e = cudaMemPoolCreate(&p, &props);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolCreate(K-part workspace)");
    unsigned long long keep = ~0ull;
    e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolSetAttribute(release threshold)");
    g_ws_pool[dev] = p;
  }
  *pool = g_ws_pool[dev];
  return QLIN_OK;
}

int run_prefill_w4(int epi, const GemvArgs& a, int half_tiles, cudaStream_t st) {
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  GemmW4Args g;
  memset(&g, 0, sizeof(g));
  if (int r = make_map(&g.ta, a.a_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.K, a.M, a.K, 128, kGmRows, true)) return r;
  const uint32_t nsr = g4_scale_rows(a.wgrp);
  bool vec = aligned(a.out, 16) && a.ldo % 8 == 0 && (!a.res || (aligned(a.res, 16) && a.ldr % 8 == 0));
  for (int i = 0; i < a.nseg; ++i) {
    const GemvSeg& s0 = a.seg[i];
    GemvSeg& s1 = g.seg[i];
    s1 = s0;
    if (int r = make_map(&s1.tw, s0.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, s0.n, a.K / 2, s0.n, kTileN, 64)) return r;
    if (int r = make_map(&s1.ts, s0.sp, CU_TENSOR_MAP_DATA_TYPE_UINT16, s0.n, a.K / a.wgrp, 2ull * s0.n, kTileN, nsr))
      return r;
    if (s0.zp) {
      if (int r = make_map(&s1.tz, s0.zp, CU_TENSOR_MAP_DATA_TYPE_UINT8, s0.n, a.K / a.wgrp, s0.n, kTileN, nsr))
        return r;
    }
    vec = vec && s0.out_col % 8 == 0;
  }
  g.nseg = a.nseg;
  g.half_tiles = half_tiles;
  g.a_s = a.a_s;
  g.M = a.M;
  g.K = a.K;
  g.wgrp = a.wgrp;
  g.out = a.out;
  g.ldo = a.ldo;
  g.res = a.res;
  g.ldr = a.ldr;
  g.vec_out = vec ? 1 : 0;
  g.out_q = a.out_q;
  g.out_s = a.out_s;
  g.n_q = a.n_q;
  g.fault = di.fault;
  if (epi != kEpiOut) g.half_tiles = 2 * half_tiles;  // (gate tile, up tile) pairs
  const long long mtiles = (a.M + kGmRows - 1) / kGmRows;
  int hs = epi == kEpiOut ? 1 : 2;  // as for W8 (config-3 W4: M = 2048 450 -> 378 us, M = 512 156 -> 107 us)
#ifdef QLIN_TUNING
  if (epi == kEpiOut && tune_half() == 2) hs = 2;
#endif
  const long long tiles = mtiles * ((g.half_tiles + hs - 1) / hs);
  int grid = static_cast<int>(tiles < di.sms ? tiles : di.sms);
  // K parts: a launch with fewer tiles than SMs (a column shard of a
  // tensor-parallel layer, a mid-size M) gives each tile up to sms / tiles
  // CTAs over disjoint stage ranges, at least two 128-K stages each.
  const int nstage = (a.K / kGroup + 1) / 2;
  long long kp = tiles < di.sms ? di.sms / tiles : 1;
  if (kp > nstage / 2) kp = nstage / 2;
  if (kp > kG4MaxParts) kp = kG4MaxParts;
#ifdef QLIN_TUNING
  if (tune_kparts() > 0) kp = tune_kparts() < nstage ? tune_kparts() : nstage;
  if (kp > kG4MaxParts) kp = kG4MaxParts;
#endif
  // every part's rows of one CTA are summed in the stage ring
  while (kp > 1 && kp * ((128 + kp - 1) / kp) * hs * 128 * 4 > static_cast<long long>(kG4Stages) * kG4StageAligned)
    --kp;
  if (kp < 1) kp = 1;
  void* ws = nullptr;
  cudaMemPool_t pool = nullptr;
  if (kp > 1) {
    if (int r = ws_pool(di.dev, &pool)) return r;
    const size_t ws_bytes = static_cast<size_t>(tiles) * kp * 128 * hs * 128 * 4;
    const size_t cnt_bytes = static_cast<size_t>(tiles) * 4;
    cudaError_t e = cudaMallocFromPoolAsync(&ws, ws_bytes + cnt_bytes, pool, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocFromPoolAsync(K-part workspace)");
    g.ws = static_cast<float*>(ws);
    g.cnt = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + ws_bytes);
    e = cudaMemsetAsync(g.cnt, 0, cnt_bytes, st);
    if (e != cudaSuccess) {
      cudaFreeAsync(ws, st);
      return cuda_fail(e, "cudaMemsetAsync(K-part counters)");
    }
    grid = static_cast<int>(tiles * kp);  // one CTA per (tile, part), all resident
  }
  g.kparts = static_cast<int>(kp);
  int r;
  if (epi != kEpiOut) {
    r = launch_prefill_w4<kEpiSiluQuant>(g, grid, st);
  } else {
#ifdef QLIN_TUNING
    if (hs == 2) r = launch_prefill_w4<kEpiOut>(g, grid, st);
    else
#endif
    r = launch_prefill_w4<kEpiOut, 1>(g, grid, st);
  }
  if (ws) {
    cudaError_t e = cudaFreeAsync(ws, st);
    if (r == QLIN_OK && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync(K-part workspace)");
  }
  return r;
}

// Fills the split / ring fields of `a`, then launches.
// Between 33 and prefill_min_m() rows the small-M kernel streams every weight
// once per row block (16 rows for W4, 32 for W8), while the tensor-core GEMM
// streams it once -- but it has no K split, so it needs many output tiles to
// fill the GPU.  Measured on B200 (one call, M = 64): config-5 fused W4 gate/up
// (K = 5120, 136 GEMM tiles) 418 us small-M vs 219 us GEMM; W8 K = 5120, N =
// 17408 (68 tiles) 82 vs 67 us; with 48 or fewer tiles the small-M kernel
// wins (config-2 gate/up 67 vs 102 us, config-5 down 420 vs 671 us).
// Long-K W4 plain outputs with at least kMidGemmLongKTiles column tiles take the
// GEMM too: its K parts spread a few tiles over the SMs while the small-M
// kernel re-streams the long weight rows per 16-row block.  Measured at M = 64
// (config-5 down 17408 -> 5120 and its column shards of 2, 4, 8 GPUs, us,
// small-M vs GEMM): 143 vs 103, 81 vs 55, 40 vs 37, 22 vs 33.
constexpr int kMidGemmMinM = 33;
constexpr long long kMidGemmMinTiles = 64;
constexpr int64_t kMidGemmLongK = 8192;
constexpr int kMidGemmLongKTiles = 8;
bool mid_m_takes_gemm(int wb, int epi, int64_t M, int64_t K, int tiles) {
  if (M < kMidGemmMinM) return false;
  const long long gemm_tiles = ((M + kGmRows - 1) / kGmRows) * (epi == kEpiOut ? (tiles + 1) / 2 : tiles);
  if (wb == 4 && epi == kEpiOut && K >= kMidGemmLongK && tiles >= kMidGemmLongKTiles) return true;  // (W4 GEMM: K parts)
  return gemm_tiles >= kMidGemmMinTiles;
}

int smem_optin(const void* kern, size_t bytes, std::atomic<unsigned long long>& done);

// ---------------------------------------------------------------- dp4a GEMV (decode rows)
// Per-CTA shared memory that keeps two CTAs on an SM (this launch and the
// next one's, which streams its weights under programmatic dependent launch).
constexpr uint32_t kDpBudget = 110 * 1024;
// Rows it serves: 1-2 (any weights), 3-4 (W4, short launches: plan_dp).  Its
// dp4a work grows with M while the tensor-core kernel's MMA count does not;
// measured on B200 (graph replay, rotating weights, us, dp4a vs tcgen05, M =
// 1): W4 gate/up 2048->2x6144 4.6 vs 8.6, down 6144->2048 3.8 vs 5.7, o 2.6
// vs 3.8, qkv 3.0 vs 4.6, W8 2048->6144 3.3 vs 3.9, W8 down 4.0 vs 5.6.

int dp_mr(int64_t M) { return M <= 1 ? 1 : M <= 2 ? 2 : 4; }

struct DpPlan {
  int split = 0, kout = 1, ring = 0, gmax = 0;
  size_t smem = 0;
};

// Resident plan: the smallest cluster split whose CTAs cover the SMs and
// whose resident weights fit the budget, at most the portable cluster size
// of 8.  For W8 a plan is taken only if all its CTAs are resident at once
// (at most two per SM: a second wave would request its weights only after
// the dependency) and its clusters are not of 7 CTAs (which pack poorly into
// B200's GPCs).  Measured: W8 gate/up 2048->2x6144 at M = 1 needs split 7
// (336 CTAs) to fit and took 7.9 us against 6.6 on the tensor-core kernel;
// the 1187-tile W8 lm_head (split 3, 3561 CTAs) 61 against 56 us.
bool plan_dp_resident(int wb, int mr, int ns, int K, int wgrp, int tiles, int sms, DpPlan* pl) {
  const int G = K / kGroup;
  DpPlan best;
  for (int s = 1; s <= 8 && s <= G; ++s) {
    const int gmax = (G + s - 1) / s;
    const DpLayout L = dp_layout(wb, mr, ns, wgrp, gmax, s, 0);
    if (L.total > kDpBudget) continue;
    best.split = s, best.gmax = gmax, best.smem = L.total;
    if (static_cast<long long>(tiles) * s >= sms) break;
  }
  if (best.split == 0) return false;
  if (wb == 8 && (best.split == 7 || static_cast<long long>(tiles) * best.split > 2ll * sms)) return false;
  *pl = best;
  return true;
}

// Ring plan for launches whose weights do not fit in one resident wave: one
// wave of CTAs without clusters, a tile's K cut into `kout` parts that meet
// in the device workspace, each warp streaming its items through a ring of
// slots.  Parts per tile are chosen so that the busiest SM streams the fewest
// groups (CTAs per SM x groups per CTA), at most two CTAs per SM (the
// kernel's register bound; shared memory 200 / 110 KB), ties to fewer parts.
bool plan_dp_ring(int wb, int mr, int ns, int K, int wgrp, int tiles, int sms, DpPlan* pl) {
  const int G = K / kGroup;
  long long best_w = -1;
  for (int P = 1; P <= G; ++P) {
    const long long ctas = static_cast<long long>(tiles) * P;
    const long long per_sm = (ctas + sms - 1) / sms;
    if (per_sm > 2) break;
    if (P > 1 && (tiles > kDpWsTiles || ctas * ns * mr * kTileN > kDpWsFloats)) break;
    const uint32_t budget = (per_sm == 1 ? 200u : 110u) * 1024u;
    const int gmax = (G + P - 1) / P;
    int ring = 0;
    for (int r = 8; r >= 2 && ring == 0; --r)
      if (dp_layout(wb, mr, ns, wgrp, gmax, 1, r).total <= budget) ring = r;
    if (ring == 0) continue;
    const int per_warp = (gmax * ns + kRgWarps - 1) / kRgWarps;
    if (ring > per_warp) ring = per_warp < 2 ? 2 : per_warp;
    const long long w = per_sm * gmax;
    if (best_w < 0 || w < best_w) {
      best_w = w;
      pl->split = 1;
      pl->kout = P;
      pl->ring = ring;
      pl->gmax = gmax;
      pl->smem = dp_layout(wb, mr, ns, wgrp, gmax, 1, ring).total;
    }
  }
  return best_w >= 0;
}

// dp plan of a launch, or false (the tensor-core kernel takes it).  W4 takes
// the resident plan when its CTAs fit one wave (at most two per SM), a ring
// plan otherwise.  Measured on B200 (graph replay, rotating weights, us, M = 1,
// ring / resident over several waves / tensor cores): config-5 W4 gate/up
// 5120->2x17408 30.1 / 29.5 / 42.7, its column shards of 2, 4, 8 GPUs 17.8 /
// 17.2 / 22.1, 10.1 / 10.1 / 12.3, 5.9 / 5.9 / 9.1; config-5 down 17408->5120
// (no resident plan) 14.4 / - / 25.5, shards 11.9 / - / 16.0, 9.3 / - / 15.1,
// 8.8 / - / 13.4.  W8 takes resident plans only (above).
bool plan_dp_uncached(int wb, int mr, int ns, int K, int wgrp, int tiles, int sms, DpPlan* pl) {
  DpPlan res;
  const bool has_res = plan_dp_resident(wb, mr, ns, K, wgrp, tiles, sms, &res);
  const bool one_wave = has_res && static_cast<long long>(tiles) * res.split <= 2ll * sms;
  if (mr > 2) {
    // 3-4 rows: W4 only, resident single-wave plans with at most two items
    // per warp (the dot work grows with the rows, the MMA count does not).
    // Measured on B200 (graph replay, us, dp4a vs tcgen05, M = 4): config-2
    // W4 gate/up 8.2 vs 10.0 (two items per warp), down 6.2 vs 6.8, o 3.9 vs
    // 4.0, qkv 4.9 vs 4.7; config-5 gate/up shards (2.5 items per warp) 19.8
    // vs 16.9 and 18.3 vs 12.2; W8 config 1 4.7 vs 4.0.
    if (tune_dp_m4() == 0) {
      if (wb != 4) return false;
      if (has_res && one_wave && res.gmax * ns <= 2 * kRgWarps) {
        *pl = res;
        return true;
      }
      // long-K launches of one stream with no resident plan: the ring, with
      // K parts over the SMs (the tensor-core kernel caps the K split at the
      // cluster size).  Config-5 down 17408 -> 5120 and its 2-, 4-, 8-GPU
      // shards at M = 4: 25.1 / 16.4 / 16.1 / 17.7 us against 30.2 / 16.5 /
      // 19.7 / 18.0 on the tensor cores.
      if (ns == 1 && !has_res && tune_dp_m4ring()) return plan_dp_ring(wb, mr, ns, K, wgrp, tiles, sms, pl);
      return false;
    }
  }
  const int mode = tune_dp_stream();
  if (has_res && (mode == 0 || (mode == 1 && one_wave))) {
    *pl = res;
    return true;
  }
  DpPlan ring;
  if (mode != 0 && (wb == 4 || mode == 2) && plan_dp_ring(wb, mr, ns, K, wgrp, tiles, sms, &ring)) {
    *pl = ring;
    return true;
  }
  if (has_res) {
    *pl = res;
    return true;
  }
  return false;
}

bool plan_dp(int wb, int mr, int ns, int K, int wgrp, int tiles, int sms, DpPlan* pl) {
  static std::mutex mu;
  static std::unordered_map<TcKey, DpPlan, TcKeyHash> cache;  // (M field: rows of the instance)
  const TcKey k{wb, ns, K, wgrp, tiles, sms, 0, mr};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(k);
    if (it != cache.end()) {
      *pl = it->second;
      return pl->split > 0;
    }
  }
  DpPlan got;
  if (!plan_dp_uncached(wb, mr, ns, K, wgrp, tiles, sms, &got)) got = DpPlan{};
  {
    std::lock_guard<std::mutex> g(mu);
    if (cache.size() >= kPlanCache) cache.clear();
    cache.emplace(k, got);
  }
  *pl = got;
  return got.split > 0;
}

// Workspace slot of the next cross-cluster launch.
int dp_ws_next_slot() {
  static std::atomic<unsigned> next{0};
  return static_cast<int>(next.fetch_add(1u) % kDpWsSlots);
}

template <int WB, int MR, int EPI>
int launch_dp_t(const DpArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = dp_gemv_kernel<WB, MR, EPI>;
  static std::atomic<unsigned long long> done{0};
  if (int r = smem_optin(reinterpret_cast<const void*>(kern), 201 * 1024, done)) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kRgThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = grid.x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = tune_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(dp_gemv)");
  return QLIN_OK;
}

template <int WB, int EPI>
int launch_dp_mr(int mr, const DpArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
  if (mr == 1) return launch_dp_t<WB, 1, EPI>(a, grid, smem, st);
#ifdef QLIN_TUNING
  if (mr == 4) return launch_dp_t<WB, 4, EPI>(a, grid, smem, st);
#else
  if constexpr (WB == 4) {
    if (mr == 4) return launch_dp_t<WB, 4, EPI>(a, grid, smem, st);
  }
#endif
  return launch_dp_t<WB, 2, EPI>(a, grid, smem, st);
}

// Launches the dp kernel if the shape fits it; *taken = false otherwise.
int run_dp(int wb, int epi, const GemvArgs& a, int tiles, cudaStream_t st, bool* taken) {
  *taken = false;
  if (a.M > tune_dp_maxm() || a.M < 1 || tiles > 65535) return QLIN_OK;
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  const int mr = dp_mr(a.M);
  const int ns = epi == kEpiOut ? 1 : 2;
  DpPlan pl;
  if (!plan_dp(wb, mr, ns, a.K, a.wgrp, tiles, di.sms, &pl)) return QLIN_OK;
  DpArgs d;
  memset(&d, 0, sizeof(d));
  const uint32_t nsr = (wb == 4 && a.wgrp == 32) ? 2 : 1;
  for (int i = 0; i < a.nseg; ++i) {
    const GemvSeg& s0 = a.seg[i];
    d.seg[i] = s0;
    if (wb == 8) {
      if (int r = make_map(&d.tw[i], s0.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, s0.n, a.K, s0.n, kTileN, 64)) return r;
    } else {
      if (int r = make_map(&d.tw[i], s0.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, s0.n, a.K / 2, s0.n, kTileN, 32)) return r;
      if (int r = make_map(&d.ts[i], s0.sp, CU_TENSOR_MAP_DATA_TYPE_UINT16, s0.n, a.K / a.wgrp, 2ull * s0.n, kTileN,
                           nsr))
        return r;
      if (s0.zp) {
        if (int r = make_map(&d.tz[i], s0.zp, CU_TENSOR_MAP_DATA_TYPE_UINT8, s0.n, a.K / a.wgrp, s0.n, kTileN, nsr))
          return r;
      }
    }
  }
  d.nseg = a.nseg;
  d.a_q = a.a_q;
  d.a_s = a.a_s;
  d.M = a.M;
  d.K = a.K;
  d.wgrp = a.wgrp;
  d.split = pl.split;
  d.gmax = pl.gmax;
  d.ring = pl.ring;
  d.kout = pl.kout;
  d.ws_slot = pl.kout > 1 ? dp_ws_next_slot() : 0;
  d.tl_slot = tl_next_slot();
  d.out = a.out;
  d.ldo = a.ldo;
  d.res = a.res;
  d.ldr = a.ldr;
  d.out_q = a.out_q;
  d.out_s = a.out_s;
  d.n_q = a.n_q;
  if (a.peer) d.peer = *static_cast<const DpPeer*>(a.peer);
  d.fault = di.fault;
  *taken = true;
  const dim3 grid(pl.split, tiles, pl.kout);
  const size_t smem = pl.smem;
  if (wb == 8) {
    switch (epi) {
      case kEpiOut: return launch_dp_mr<8, kEpiOut>(mr, d, grid, smem, st);
      case kEpiSiluBf16: return launch_dp_mr<8, kEpiSiluBf16>(mr, d, grid, smem, st);
      default: return launch_dp_mr<8, kEpiSiluQuant>(mr, d, grid, smem, st);
    }
  }
  switch (epi) {
    case kEpiOut: return launch_dp_mr<4, kEpiOut>(mr, d, grid, smem, st);
    default: return launch_dp_mr<4, kEpiSiluQuant>(mr, d, grid, smem, st);
  }
}

int run_gemv(int wb, int epi, GemvArgs& a, int tiles, cudaStream_t st) {
  if (a.peer) {
    // the column-split layer's down projection with its gathers inside: the dp kernel only
    bool taken = false;
    if (int r = run_dp(wb, epi, a, tiles, st, &taken)) return r;
    if (!taken) return fail(QLIN_ERR_UNSUPPORTED, "no decode-row plan for this shape");
    return QLIN_OK;
  }
  const bool gemm = a.M >= prefill_min_m() || mid_m_takes_gemm(wb, epi, a.M, a.K, tiles);
  if (wb == 8 && gemm) return run_prefill_w8(epi, a, tiles, st);
  if (wb == 4 && gemm && a.wgrp % 64 == 0) return run_prefill_w4(epi, a, tiles, st);
  if (use_dp()) {
    bool taken = false;
    if (int r = run_dp(wb, epi, a, tiles, st, &taken)) return r;
    if (taken) return QLIN_OK;
  }
  return run_tc(wb, epi, a, tiles, st);
}

// ---------------------------------------------------------------- argument checks
int check_common(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, int64_t N) {
  if (M < 0 || K < 0 || N < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "negative size");
  if (M > (1ll << 30) || K > (1ll << 30) || N > (1ll << 30)) return fail(QLIN_ERR_SHAPE, "size too large");
  if (K == 0 || K % kGroup != 0) return fail(QLIN_ERR_SHAPE, "K=%lld must be a positive multiple of 64", (long long)K);
  if (M > 0 && (!a_q || !a_s)) return fail(QLIN_ERR_INVALID_ARGUMENT, "null activation pointer");
  if (!aligned(a_q, 16)) return fail(QLIN_ERR_ALIGNMENT, "a_q must be 16-byte aligned");
  if (!aligned(a_s, 4)) return fail(QLIN_ERR_ALIGNMENT, "a_s must be 4-byte aligned");
  return QLIN_OK;
}

int check_n(int64_t N) {
  if (N % 16 != 0) return fail(QLIN_ERR_ALIGNMENT, "N=%lld must be a multiple of 16", (long long)N);
  return QLIN_OK;
}

int check_wgrp(int64_t K, int64_t wgrp) {
  if (!(wgrp == 32 || (wgrp >= 64 && wgrp % 64 == 0)) || K % wgrp != 0)
    return fail(QLIN_ERR_SHAPE, "W4 group size %lld unsupported for K=%lld (32 or a multiple of 64)",
                (long long)wgrp, (long long)K);
  return QLIN_OK;
}

int seg_w8(GemvSeg& s, const int8_t* w, const float* bs, int64_t K, int64_t n) {
  if (!w || !bs) return fail(QLIN_ERR_INVALID_ARGUMENT, "null W8 weight/scale pointer");
  if (!aligned(w, 16)) return fail(QLIN_ERR_ALIGNMENT, "W8 weight must be 16-byte aligned");
  if (!aligned(bs, 4)) return fail(QLIN_ERR_ALIGNMENT, "W8 scales must be 4-byte aligned");
  // 128-byte swizzle: the tile lands in the canonical MN-major layout that
  // tcgen05.mma reads.
  if (int r = make_map(&s.tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, K, n, kTileN, 64, true)) return r;
  s.w = w;
  s.bs = bs;
  s.n = static_cast<int>(n);
  s.has_z = 0;
  return QLIN_OK;
}

int seg_w4(GemvSeg& s, const uint8_t* w, const void* sc, const uint8_t* z, int64_t K, int64_t n,
           int64_t wgrp) {
  if (!w || !sc) return fail(QLIN_ERR_INVALID_ARGUMENT, "null W4 weight/scale pointer");
  if (!aligned(w, 16) || !aligned(sc, 16) || (z && !aligned(z, 16)))
    return fail(QLIN_ERR_ALIGNMENT, "W4 weight/scale/zero tensors must be 16-byte aligned");
  const uint32_t nsr = wgrp == 32 ? 2 : 1;
  // 128-byte swizzle for the tcgen05 kernel, which unpacks half of each
  // group in place into the MMA operand layout.
  if (int r = make_map(&s.tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, K / 2, n, kTileN, 32, true)) return r;
  if (int r = make_map(&s.ts, sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, n, K / wgrp, 2 * n, kTileN, nsr)) return r;
  if (z) {
    if (int r = make_map(&s.tz, z, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, K / wgrp, n, kTileN, nsr)) return r;
  }
  s.bs = nullptr;
  s.n = static_cast<int>(n);
  s.has_z = z ? 1 : 0;
  s.w = w;
  s.sp = sc;
  s.zp = z;
  return QLIN_OK;
}

int tiles_of(int64_t n) { return static_cast<int>((n + kTileN - 1) / kTileN); }

// Device addresses of one GPU's static gather scratch.  In host code the
// names g_static_* only stand in for the device variables, so the addresses
// are looked up once per device, with that device current.
struct StaticGather {
  bool ready;
  uint8_t* buf;
  unsigned* arrive;
  unsigned* expected;
};
StaticGather g_static[kMaxDevices];
std::mutex g_static_mu;

int static_gather_setup(int dev) {  // with g_static_mu held and `dev` current
  StaticGather& g = g_static[dev];
  if (g.ready) return QLIN_OK;
  void *b = nullptr, *a = nullptr, *x = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&b, g_static_gather);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static gather buffer)");
  if ((e = cudaGetSymbolAddress(&a, g_static_arrive)) != cudaSuccess)
    return cuda_fail(e, "cudaGetSymbolAddress(static arrival counters)");
  if ((e = cudaGetSymbolAddress(&x, g_static_expected)) != cudaSuccess)
    return cuda_fail(e, "cudaGetSymbolAddress(static expected counts)");
  g.buf = static_cast<uint8_t*>(b);
  g.arrive = static_cast<unsigned*>(a);
  g.expected = static_cast<unsigned*>(x);
  g.ready = true;
  return QLIN_OK;
}

// Grid of the gather kernel: depends on the sizes only, so every rank (which
// passes the same sizes) launches the same number of CTAs -- each CTA adds
// one arrival on every rank.
int peer_ctas(long long units16) {
  long long ctas = (units16 + kPeerThreads * 4 - 1) / (kPeerThreads * 4);
  if (ctas < 1) ctas = 1;
  if (ctas > kPeerMaxCtas) ctas = kPeerMaxCtas;
  return static_cast<int>(ctas);
}

int peer_buffers(PeerGatherArgs& a, void* const* bufs, void* const* arrive, int world) {
  for (int q = 0; q < world; ++q) {
    if (!bufs[q] || !arrive[q] || !aligned(bufs[q], 16) || !aligned(arrive[q], 4))
      return fail(QLIN_ERR_ALIGNMENT, "peer buffer %d is null or misaligned", q);
    a.bufs[q] = static_cast<uint8_t*>(bufs[q]);
    a.arrive[q] = static_cast<unsigned*>(arrive[q]);
  }
  return QLIN_OK;
}

int peer_launch(const PeerGatherArgs& a, int ctas, cudaStream_t st) {
  if (int r = prefer_shared(reinterpret_cast<const void*>(peer_allgather_kernel))) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kPeerThreads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, peer_allgather_kernel, a);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(peer_allgather)");
  return QLIN_OK;
}

// ---------------------------------------------------------------- activation producers (kernels/norm.py)
int prod_launch(const void* kern, dim3 grid, void** args, cudaStream_t st) {
  if (int r = prefer_shared(kern)) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kProdThreads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelExC(&cfg, kern, args);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(producer)");
  return QLIN_OK;
}

int check_rows(int64_t M, int64_t K, const char* what) {
  if (M < 0 || K < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "%s: negative size", what);
  if (M > 65535 * 64) return fail(QLIN_ERR_SHAPE, "%s: M=%lld too large", what, (long long)M);
  return QLIN_OK;
}

// ---------------------------------------------------------------- decode-step neighbours
int dec_launch(const void* kern, dim3 grid, dim3 block, size_t smem, int cluster, void** args, cudaStream_t st) {
  if (int r = prefer_shared(kern)) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelExC(&cfg, kern, args);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(decode neighbour)");
  return QLIN_OK;
}

// Opt a kernel in to `bytes` of dynamic shared memory once per device.
int smem_optin(const void* kern, size_t bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(smem)");
    if (int r = prefer_shared(kern)) return r;
    done.fetch_or(bit);
  }
  return QLIN_OK;
}

template <int G, int E, bool INT8>
int launch_attn_decode(AttnDecodeArgs& a, int S, int nkv, int B, cudaStream_t st) {
  static std::atomic<unsigned long long> done{0};
  const void* kern = reinterpret_cast<const void*>(attn_decode_kernel<G, E, INT8>);
  const size_t smem = attn_decode_smem(G, E);
  if (int r = smem_optin(kern, smem, done)) return r;
  void* args[] = {&a};
  return dec_launch(kern, dim3(S, nkv, B), dim3(kDecThreads), smem, S, args, st);
}

template <int E, bool INT8>
int attn_decode_g(int G, AttnDecodeArgs& a, int S, int nkv, int B, cudaStream_t st) {
  switch (G) {
    case 1: return launch_attn_decode<1, E, INT8>(a, S, nkv, B, st);
    case 2: return launch_attn_decode<2, E, INT8>(a, S, nkv, B, st);
    case 4: return launch_attn_decode<4, E, INT8>(a, S, nkv, B, st);
    case 8: return launch_attn_decode<8, E, INT8>(a, S, nkv, B, st);
    default: return fail(QLIN_ERR_SHAPE, "attn_decode: %d query heads per KV head (1, 2, 4 or 8)", G);
  }
}
}  // namespace
}  // namespace qlin

using namespace qlin;

// =====================================================================================
extern "C" {

int qlin_version(void) { return kVersion; }

const char* qlin_status_string(int s) {
  switch (s) {
    case QLIN_OK: return "ok";
    case QLIN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case QLIN_ERR_SHAPE: return "unsupported shape";
    case QLIN_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case QLIN_ERR_UNSUPPORTED: return "unsupported";
    case QLIN_ERR_CUDA: return "CUDA error";
    case QLIN_ERR_DEVICE_FAULT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

const char* qlin_last_error(void) { return g_err; }

int qlin_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return fail(QLIN_ERR_INVALID_ARGUMENT, "null argument");
  CUdeviceptr base = 0;
  if (int r = address_range(ptr, &base)) return r;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == QLIN_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return QLIN_OK;
}

int qlin_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "bad IPC open arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr = static_cast<uint8_t*>(base) + offset;
  return QLIN_OK;
}

int qlin_ipc_close(void* ptr, int64_t offset) {
  if (!ptr) return QLIN_OK;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return QLIN_OK;
}

int qlin_dev_alloc(int64_t bytes, void** ptr) {
  if (bytes <= 0 || !ptr) return fail(QLIN_ERR_INVALID_ARGUMENT, "bad allocation request");
  cudaError_t e = cudaMalloc(ptr, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  e = cudaMemset(*ptr, 0, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset");
  return QLIN_OK;
}

int qlin_dev_free(void* ptr) {
  if (!ptr) return QLIN_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree");
  return QLIN_OK;
}

int qlin_peer_allgather(void* const* bufs, void* const* arrive, void* expected, const void* src,
                        int64_t shard_bytes, int world, int rank, void* dst, void* stream) {
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "world %d / rank %d", world, rank);
  if (!bufs || !arrive || !expected || !src) return fail(QLIN_ERR_INVALID_ARGUMENT, "null argument");
  if (shard_bytes <= 0 || shard_bytes % 16 != 0)
    return fail(QLIN_ERR_SHAPE, "shard of %lld bytes is not a positive multiple of 16", (long long)shard_bytes);
  if (!aligned(src, 16)) return fail(QLIN_ERR_ALIGNMENT, "source must be 16-byte aligned");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  PeerGatherArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = peer_buffers(a, bufs, arrive, world)) return r;
  a.expected = static_cast<unsigned*>(expected);
  // one row of shard_bytes: rank q's shard at byte q * shard_bytes
  a.part[0] = PeerPart{static_cast<const uint8_t*>(src), 0, 1, shard_bytes, 0, 0, 16};
  a.nparts = 1;
  a.world = world;
  a.rank = rank;
  a.fault = di.fault;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int r = peer_launch(a, peer_ctas(shard_bytes / 16), st)) return r;
  if (dst) {
    cudaError_t e = cudaMemcpyAsync(dst, bufs[rank], static_cast<size_t>(shard_bytes) * world,
                                    cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(gathered)");
  }
  return QLIN_OK;
}

int qlin_peer_allgather_fenced(void* const* bufs, void* const* arrive, void* expected, const qlin_gather_part* parts,
                               int nparts, int world, int rank, void* stream) {
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "world %d / rank %d", world, rank);
  if (!bufs || !arrive || !expected || !parts) return fail(QLIN_ERR_INVALID_ARGUMENT, "null argument");
  if (nparts < 1 || nparts > kPeerMaxParts)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "%d parts (1 to %d)", nparts, kPeerMaxParts);
  if (!aligned(expected, 4)) return fail(QLIN_ERR_ALIGNMENT, "expected counts must be 4-byte aligned");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  PeerGatherArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = peer_buffers(a, bufs, arrive, world)) return r;
  long long units16 = 0;
  for (int i = 0; i < nparts; ++i) {
    const qlin_gather_part& q = parts[i];
    if (!q.src || q.rows < 1 || q.row_bytes < 4 || q.src_ld < 0 || q.dst_off < 0 || q.dst_ld < 0)
      return fail(QLIN_ERR_INVALID_ARGUMENT, "part %d: null source or bad size", i);
    if (q.rows > 1 && (q.src_ld < q.row_bytes || q.dst_ld < static_cast<int64_t>(world) * q.row_bytes))
      return fail(QLIN_ERR_SHAPE, "part %d: row strides overlap the rows / the ranks' slots", i);
    auto all_mult = [&](int u) {
      return q.row_bytes % u == 0 && q.src_ld % u == 0 && q.dst_off % u == 0 && q.dst_ld % u == 0 &&
             aligned(q.src, u);
    };
    const int unit = all_mult(16) ? 16 : all_mult(4) ? 4 : 0;
    if (!unit) return fail(QLIN_ERR_ALIGNMENT, "part %d: sizes, strides and addresses must be multiples of 4", i);
    a.part[i] = PeerPart{static_cast<const uint8_t*>(q.src), q.src_ld, q.rows, q.row_bytes, q.dst_off, q.dst_ld,
                         unit};
    units16 += (q.rows * q.row_bytes + 15) / 16;
  }
  a.nparts = nparts;
  a.expected = static_cast<unsigned*>(expected);
  a.world = world;
  a.rank = rank;
  a.fault = di.fault;
  // large shards: up to one CTA per SM, about 8 16-byte units per thread
  long long ctas = (units16 + kPeerThreads * 8 - 1) / (kPeerThreads * 8);
  if (ctas > di.sms) ctas = di.sms;
  if (ctas < 1) ctas = 1;
  return peer_launch(a, static_cast<int>(ctas), static_cast<cudaStream_t>(stream));
}

// Flagged-word exchange layout of `parts`: per part its unit (8 data bytes
// per 16-byte store, or 4 per 8-byte store) and its offset in a sender slot.
// Depends on the sizes only, so every rank (same sizes) gets the same layout.
int ll_layout(const qlin_gather_part* parts, int nparts, int world, LlGatherArgs* a) {
  if (world < 1 || world > kPeerMax) return fail(QLIN_ERR_INVALID_ARGUMENT, "world %d (1 to %d)", world, kPeerMax);
  if (!parts) return fail(QLIN_ERR_INVALID_ARGUMENT, "null parts");
  if (nparts < 1 || nparts > kLlMaxParts)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "%d parts (1 to %d)", nparts, kLlMaxParts);
  long long off = 0, units = 0;
  for (int i = 0; i < nparts; ++i) {
    const qlin_gather_part& q = parts[i];
    if (q.rows < 1 || q.row_bytes < 4 || q.src_ld < 0 || q.dst_off < 0 || q.dst_ld < 0)
      return fail(QLIN_ERR_INVALID_ARGUMENT, "part %d: bad size", i);
    if (q.rows > 1 && (q.src_ld < q.row_bytes || q.dst_ld < static_cast<int64_t>(world) * q.row_bytes))
      return fail(QLIN_ERR_SHAPE, "part %d: row strides overlap the rows / the ranks' slots", i);
    auto mult = [&](int u) { return q.row_bytes % u == 0 && q.dst_off % u == 0 && q.dst_ld % u == 0; };
    const int unit = mult(8) ? 8 : mult(4) ? 4 : 0;
    if (!unit) return fail(QLIN_ERR_ALIGNMENT, "part %d: row bytes and destination offsets must be multiples of 4", i);
    LlPart& p = a->part[i];
    p.src = static_cast<const uint8_t*>(q.src);
    p.src_ld = q.src_ld;
    p.rows = q.rows;
    p.row_bytes = q.row_bytes;
    p.dst_off = q.dst_off;
    p.dst_ld = q.dst_ld;
    p.ll_off = off;
    p.first = units;
    p.unit = unit;
    const long long n = q.rows * (q.row_bytes / unit);
    units += n;
    off += (n * 2 * unit + 15) / 16 * 16;
  }
  a->nparts = nparts;
  a->units = units;
  a->slot_bytes = off;
  return QLIN_OK;
}

int qlin_peer_ll_bytes(const qlin_gather_part* parts, int nparts, int world, int64_t* bytes) {
  if (!bytes) return fail(QLIN_ERR_INVALID_ARGUMENT, "null result");
  LlGatherArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = ll_layout(parts, nparts, world, &a)) return r;
  *bytes = 2LL * world * a.slot_bytes;
  return QLIN_OK;
}

static int ll_gather(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts, int nparts, int world,
              int rank, void* dst, int mode, void* state2, void* stream);

int qlin_peer_allgather_ll(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts,
                           int nparts, int world, int rank, void* dst, void* stream) {
  return ll_gather(ll, ll_bytes, state, parts, nparts, world, rank, dst, 0, nullptr, stream);
}

int qlin_peer_ll_send(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts, int nparts,
                      int world, int rank, void* stream) {
  return ll_gather(ll, ll_bytes, state, parts, nparts, world, rank, nullptr, 1, nullptr, stream);
}

int qlin_peer_ll_recv(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts, int nparts,
                      int world, int rank, void* dst, void* state2, void* stream) {
  return ll_gather(ll, ll_bytes, state, parts, nparts, world, rank, dst, 2, state2, stream);
}

static int ll_gather(void* const* ll, int64_t ll_bytes, void* state, const qlin_gather_part* parts, int nparts, int world,
              int rank, void* dst, int mode, void* state2, void* stream) {
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "world %d / rank %d", world, rank);
  if (!ll || !state || !parts || (!dst && mode != 1)) return fail(QLIN_ERR_INVALID_ARGUMENT, "null argument");
  if (!aligned(state, 4) || !aligned(state2, 4)) return fail(QLIN_ERR_ALIGNMENT, "state must be 4-byte aligned");
  LlGatherArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = ll_layout(parts, nparts, world, &a)) return r;
  if (ll_bytes < 2LL * world * a.slot_bytes)
    return fail(QLIN_ERR_SHAPE, "exchange buffers of %lld bytes, %lld needed", (long long)ll_bytes,
                2LL * world * a.slot_bytes);
  for (int q = 0; q < world; ++q) {
    if (!ll[q] || !aligned(ll[q], 16)) return fail(QLIN_ERR_ALIGNMENT, "exchange buffer %d is null or misaligned", q);
    a.ll[q] = static_cast<uint8_t*>(ll[q]);
  }
  for (int i = 0; i < nparts; ++i) {
    const LlPart& p = a.part[i];
    if ((mode != 2 && (!p.src || !aligned(p.src, p.unit) || p.src_ld % p.unit != 0)) || !aligned(dst, p.unit))
      return fail(QLIN_ERR_ALIGNMENT, "part %d: source, source stride and destination must be %d-byte aligned", i,
                  p.unit);
  }
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  a.state = static_cast<unsigned*>(state);
  a.dst = static_cast<uint8_t*>(dst);
  a.world = world;
  a.rank = rank;
  a.mode = mode;
  a.state2 = static_cast<unsigned*>(state2);
  a.fault = di.fault;
  // about two received words (or sends) per thread, at most two CTAs per SM
  // (all resident: a CTA's polls wait only on other GPUs); large gathers keep
  // kLlBatch words per thread in flight
  const long long work = a.units * (mode != 0 ? world : world > 1 ? world - 1 : 1);
  long long ctas = (work + kPeerThreads * 2 - 1) / (kPeerThreads * 2);
  if (ctas > 2LL * di.sms) ctas = 2LL * di.sms;
  if (ctas < 1) ctas = 1;
  const void* kern = reinterpret_cast<const void*>(peer_ll_gather_kernel);
  if (int r = prefer_shared(kern)) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas), 1, 1);
  cfg.blockDim = dim3(kPeerThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, peer_ll_gather_kernel, a);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(peer_ll_gather)");
  return QLIN_OK;
}

int qlin_peer_allgather_static(const void* src, int64_t shard_bytes, void* dst, void* stream) {
  if (!src || !dst) return fail(QLIN_ERR_INVALID_ARGUMENT, "null argument");
  if (shard_bytes <= 0 || shard_bytes % 16 != 0)
    return fail(QLIN_ERR_SHAPE, "shard of %lld bytes is not a positive multiple of 16", (long long)shard_bytes);
  if (shard_bytes > static_cast<int64_t>(kStaticGatherBytes))
    return fail(QLIN_ERR_SHAPE, "shard of %lld bytes exceeds the static scratch limit of %lld bytes",
                (long long)shard_bytes, (long long)kStaticGatherBytes);
  if (!aligned(src, 16)) return fail(QLIN_ERR_ALIGNMENT, "source must be 16-byte aligned");
  DevInfo di;
  if (int r = device_info_noalloc(&di)) return r;
  if (int r = sticky_fault(di)) return r;
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  PeerGatherArgs a;
  memset(&a, 0, sizeof(a));
  {
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (int r = static_gather_setup(cur)) return r;
    a.bufs[0] = g_static[cur].buf;
    a.arrive[0] = g_static[cur].arrive;
    a.expected = g_static[cur].expected;
  }
  a.part[0] = PeerPart{static_cast<const uint8_t*>(src), 0, 1, shard_bytes, 0, 0, 16};
  a.nparts = 1;
  a.world = 1;
  a.rank = 0;
  a.fault = di.fault;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int r = peer_launch(a, peer_ctas(shard_bytes / 16), st)) return r;
  e = cudaMemcpyAsync(dst, a.bufs[0], static_cast<size_t>(shard_bytes), cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(gathered)");
  return QLIN_OK;
}

int qlin_plan_small_m(int wbits, int gate_up, int64_t M, int64_t K, int64_t tiles, int64_t wgrp, int sms,
                      int64_t* out) {
  if ((wbits != 8 && wbits != 4) || !out || M <= 0 || tiles <= 0 || sms < 0)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "bad plan query");
  // sms = 0: the plan a launch on the current device gets (its SM count and
  // resident-cluster capacity).
  const bool on_device = sms == 0;
  if (on_device) {
    DevInfo di;
    if (int r = device_info(&di)) return r;
    sms = di.sms;
  }
  if (K <= 0 || K % kGroup != 0 || K > (1ll << 30)) return fail(QLIN_ERR_SHAPE, "K=%lld", (long long)K);
  if (wbits == 4)
    if (int r = check_wgrp(K, wgrp)) return r;
  int mr = 0, rowblocks = 0;
  TcPlan pl{};
  if (int r = choose_tc(wbits, gate_up ? 2 : 1, M, static_cast<int>(K), wbits == 4 ? static_cast<int>(wgrp) : 64,
                        static_cast<int>(tiles > 65536 ? 65536 : tiles), sms, on_device, &mr, &rowblocks, &pl))
    return r;
  const int64_t v[10] = {pl.split, pl.gmax, pl.bs, pl.rb, pl.ab, pl.nbb, static_cast<int64_t>(pl.smem), mr,
                         pl.alias, pl.level};
  for (int i = 0; i < 10; ++i) out[i] = v[i];
  return QLIN_OK;
}

int qlin_max_active_clusters(int wbits, int gate_up, int64_t M, int split, int64_t smem, int64_t* out) {
  if ((wbits != 8 && wbits != 4) || !out || M <= 0 || split < 1 || split > kMaxCluster || smem < 0 ||
      smem > static_cast<int64_t>(kTcMaxSmem))
    return fail(QLIN_ERR_INVALID_ARGUMENT, "bad cluster query");
  const int n = active_clusters(wbits, tc_mr(wbits, M), gate_up ? 2 : 1, split, static_cast<size_t>(smem));
  if (n < 0) return fail(QLIN_ERR_CUDA, "cudaOccupancyMaxActiveClusters unavailable");
  *out = n;
  return QLIN_OK;
}

int qlin_device_fault(int clear) {
  DevInfo di;
  if (device_info_noalloc(&di) != QLIN_OK) return -1;
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_qlin_fault, sizeof(v)) != cudaSuccess) return -1;
  if (clear) {
    const unsigned z = 0;
    if (cudaMemcpyToSymbol(g_qlin_fault, &z, sizeof(z)) != cudaSuccess) return -1;
    if (di.fault_host) *di.fault_host = 0;
  }
  return static_cast<int>(v);
}

#ifdef QLIN_TUNING
// Tuning builds: copies the phase timeline ([16 slots][2048 CTAs][8] ns stamps)
// to host memory.
int qlin_debug_timeline(void* host, int64_t bytes) {
  if (!host || bytes < static_cast<int64_t>(sizeof(g_qlin_tl))) return fail(QLIN_ERR_INVALID_ARGUMENT, "buffer");
  cudaError_t e = cudaMemcpyFromSymbol(host, g_qlin_tl, sizeof(g_qlin_tl));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(timeline)");
  return QLIN_OK;
}
#endif

int qlin_set_wait_limit_ns(int64_t ns) {
  if (ns <= 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "wait limit must be positive");
  DevInfo di;
  if (int r = device_info_noalloc(&di)) return r;
  const unsigned long long v = static_cast<unsigned long long>(ns);
  cudaError_t e = cudaMemcpyToSymbol(g_qlin_wait_ns, &v, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(wait limit)");
  return QLIN_OK;
}

int qlin_gemm_i8(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const int8_t* b,
                 const float* b_s, int64_t N, void* out, int64_t ldo, const void* residual,
                 int64_t ldr, void* stream) {
  if (int r = check_common(a_q, a_s, M, K, N)) return r;
  if (int r = check_n(N)) return r;
  if (M == 0 || N == 0) return QLIN_OK;
  if (!out) return fail(QLIN_ERR_INVALID_ARGUMENT, "null out");
  if (ldo < N || (residual && ldr < N)) return fail(QLIN_ERR_SHAPE, "row stride smaller than N");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = seg_w8(a.seg[0], b, b_s, K, N)) return r;
  a.nseg = 1;
  a.a_q = a_q;
  a.a_s = a_s;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = 64;
  a.out = out;
  a.ldo = ldo;
  a.res = residual;
  a.ldr = residual ? ldr : 0;
  return run_gemv(8, kEpiOut, a, tiles_of(N), static_cast<cudaStream_t>(stream));
}

int qlin_gemm_w4(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const uint8_t* b,
                 const void* b_s, const uint8_t* b_z, int64_t N, int64_t wgrp, void* out, int64_t ldo,
                 const void* residual, int64_t ldr, void* stream) {
  if (int r = check_common(a_q, a_s, M, K, N)) return r;
  if (int r = check_n(N)) return r;
  if (int r = check_wgrp(K, wgrp)) return r;
  if (M == 0 || N == 0) return QLIN_OK;
  if (!out) return fail(QLIN_ERR_INVALID_ARGUMENT, "null out");
  if (ldo < N || (residual && ldr < N)) return fail(QLIN_ERR_SHAPE, "row stride smaller than N");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = seg_w4(a.seg[0], b, b_s, b_z, K, N, wgrp)) return r;
  a.nseg = 1;
  a.a_q = a_q;
  a.a_s = a_s;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = static_cast<int>(wgrp);
  a.out = out;
  a.ldo = ldo;
  a.res = residual;
  a.ldr = residual ? ldr : 0;
  return run_gemv(4, kEpiOut, a, tiles_of(N), static_cast<cudaStream_t>(stream));
}

int qlin_tp_gemm_w4_ll(int64_t M, int64_t K, const uint8_t* b, const void* b_s, const uint8_t* b_z, int64_t N,
                       int64_t wgrp, void* out, int64_t ldo, void* const* h_ll, int64_t h_ll_bytes, const void* h_state,
                       const qlin_gather_part* h_parts, int h_nparts, void* const* o_ll, int64_t o_ll_bytes,
                       const void* o_state, const qlin_gather_part* o_parts, int o_nparts, int world, int rank,
                       void* hq, void* hs, void* stream) {
  if (world < 1 || world > kDpPeerMax || rank < 0 || rank >= world)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "world %d / rank %d", world, rank);
  if (!h_ll || !o_ll || !h_state || !o_state || !out) return fail(QLIN_ERR_INVALID_ARGUMENT, "null argument");
  if (M < 1 || M > 4) return fail(QLIN_ERR_SHAPE, "M=%lld: the fused column-split down projection serves 1-4 rows",
                                  (long long)M);
  if (K % (128LL * world) != 0 || N % 16 != 0 || ldo < N)
    return fail(QLIN_ERR_SHAPE, "K=%lld must split into %d multiples of 128, N=%lld a multiple of 16", (long long)K,
                world, (long long)N);
  if (int r = check_wgrp(K, wgrp)) return r;
  if (!aligned(h_state, 4) || !aligned(o_state, 4) || !aligned(out, 8) || ldo % 4 != 0 || (hq && !aligned(hq, 8)) ||
      (hs && !aligned(hs, 4)))
    return fail(QLIN_ERR_ALIGNMENT, "state, out, hq or hs misaligned");
  const int64_t kloc = K / world;
  // the exchange layouts must be those of qlin_peer_allgather_ll for [codes, scales] of h and [rows] of the output
  LlGatherArgs hl, ol;
  memset(&hl, 0, sizeof(hl));
  memset(&ol, 0, sizeof(ol));
  if (int r = ll_layout(h_parts, h_nparts, world, &hl)) return r;
  if (int r = ll_layout(o_parts, o_nparts, world, &ol)) return r;
  if (h_nparts != 2 || h_parts[0].rows != M || h_parts[0].row_bytes != kloc || h_parts[1].rows != M ||
      h_parts[1].row_bytes != kloc / 64 * 4 || hl.part[0].unit != 8 || hl.part[1].unit != 8 || o_nparts != 1 ||
      o_parts[0].rows != M || o_parts[0].row_bytes != N * 2 || ol.part[0].unit != 8)
    return fail(QLIN_ERR_SHAPE, "gather parts are not h [codes, scales] and the output rows of this launch");
  if (h_ll_bytes < 2LL * world * hl.slot_bytes || o_ll_bytes < 2LL * world * ol.slot_bytes)
    return fail(QLIN_ERR_SHAPE, "exchange buffers too small");
  DpPeer pr;
  memset(&pr, 0, sizeof(pr));
  pr.rx = static_cast<const uint8_t*>(h_ll[rank]);
  pr.rx_slot = hl.slot_bytes;
  pr.rx_off_s = hl.part[1].ll_off;
  pr.rx_state = static_cast<const unsigned*>(h_state);
  pr.rx_kloc = static_cast<int>(kloc);
  pr.rx_hq = static_cast<int8_t*>(hq);
  pr.rx_hs = static_cast<float*>(hs);
  for (int q = 0; q < world; ++q) {
    if (!h_ll[q] || !o_ll[q] || !aligned(h_ll[q], 16) || !aligned(o_ll[q], 16))
      return fail(QLIN_ERR_ALIGNMENT, "exchange buffer %d is null or misaligned", q);
    pr.tx[q] = static_cast<uint8_t*>(o_ll[q]);
  }
  pr.tx_slot = ol.slot_bytes;
  pr.tx_state = static_cast<const unsigned*>(o_state);
  pr.world = world;
  pr.rank = rank;
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = seg_w4(a.seg[0], b, b_s, b_z, K, N, wgrp)) return r;
  a.nseg = 1;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = static_cast<int>(wgrp);
  a.out = out;
  a.ldo = ldo;
  a.peer = &pr;
  return run_gemv(4, kEpiOut, a, tiles_of(N), static_cast<cudaStream_t>(stream));
}

int qlin_plan_dp(int wbits, int gate_up, int64_t M, int64_t K, int64_t tiles, int64_t wgrp, int sms, int64_t* out) {
  if ((wbits != 8 && wbits != 4) || !out || M <= 0 || tiles <= 0 || sms < 0 || K <= 0)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "bad plan query");
  if (sms == 0) {
    DevInfo di;
    if (int r = launch_info(&di)) return r;
    sms = di.sms;
  }
  for (int i = 0; i < 4; ++i) out[i] = 0;
  if (M > tune_dp_maxm() || !use_dp()) return QLIN_OK;
  DpPlan pl;
  if (!plan_dp(wbits, dp_mr(M), gate_up ? 2 : 1, static_cast<int>(K), static_cast<int>(wgrp), static_cast<int>(tiles),
               sms, &pl))
    return QLIN_OK;
  out[0] = pl.split;
  out[1] = pl.kout;
  out[2] = pl.ring;
  out[3] = pl.gmax;
  return QLIN_OK;
}

int qlin_proj3(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const int8_t* w1,
               const float* s1, int64_t n1, const int8_t* w2, const float* s2, int64_t n2,
               const int8_t* w3, const float* s3, int64_t n3, void* out, int64_t ldo, void* stream) {
  const int64_t ns[3] = {n1, n2, n3};
  const int8_t* ws[3] = {w1, w2, w3};
  const float* ss[3] = {s1, s2, s3};
  const int64_t NT = n1 + n2 + n3;
  if (int r = check_common(a_q, a_s, M, K, NT)) return r;
  if (M == 0 || NT == 0) return QLIN_OK;
  if (!out) return fail(QLIN_ERR_INVALID_ARGUMENT, "null out");
  if (ldo < NT) return fail(QLIN_ERR_SHAPE, "row stride smaller than n1+n2+n3");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  int tiles = 0, col = 0, k = 0;
  for (int i = 0; i < 3; ++i) {
    if (ns[i] < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "negative segment width");
    if (ns[i] == 0) continue;
    if (int r = check_n(ns[i])) return r;
    if (int r = seg_w8(a.seg[k], ws[i], ss[i], K, ns[i])) return r;
    a.seg[k].out_col = col;
    a.seg[k].tile_begin = tiles;
    col += static_cast<int>(ns[i]);
    tiles += tiles_of(ns[i]);
    ++k;
  }
  a.nseg = k;
  a.a_q = a_q;
  a.a_s = a_s;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = 64;
  a.out = out;
  a.ldo = ldo;
  return run_gemv(8, kEpiOut, a, tiles, static_cast<cudaStream_t>(stream));
}

int qlin_proj3_w4(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const uint8_t* w1,
                  const void* s1, const uint8_t* z1, int64_t n1, const uint8_t* w2, const void* s2,
                  const uint8_t* z2, int64_t n2, const uint8_t* w3, const void* s3, const uint8_t* z3,
                  int64_t n3, int64_t wgrp, void* out, int64_t ldo, void* stream) {
  const int64_t ns[3] = {n1, n2, n3};
  const uint8_t* ws[3] = {w1, w2, w3};
  const void* ss[3] = {s1, s2, s3};
  const uint8_t* zs[3] = {z1, z2, z3};
  const int64_t NT = n1 + n2 + n3;
  if (int r = check_common(a_q, a_s, M, K, NT)) return r;
  if (int r = check_wgrp(K, wgrp)) return r;
  if (M == 0 || NT == 0) return QLIN_OK;
  if (!out) return fail(QLIN_ERR_INVALID_ARGUMENT, "null out");
  if (ldo < NT) return fail(QLIN_ERR_SHAPE, "row stride smaller than n1+n2+n3");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  int tiles = 0, col = 0, k = 0;
  for (int i = 0; i < 3; ++i) {
    if (ns[i] < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "negative segment width");
    if (ns[i] == 0) continue;
    if (int r = check_n(ns[i])) return r;
    if (int r = seg_w4(a.seg[k], ws[i], ss[i], zs[i], K, ns[i], wgrp)) return r;
    a.seg[k].out_col = col;
    a.seg[k].tile_begin = tiles;
    col += static_cast<int>(ns[i]);
    tiles += tiles_of(ns[i]);
    ++k;
  }
  a.nseg = k;
  a.a_q = a_q;
  a.a_s = a_s;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = static_cast<int>(wgrp);
  a.out = out;
  a.ldo = ldo;
  return run_gemv(4, kEpiOut, a, tiles, static_cast<cudaStream_t>(stream));
}

static int gate_up_w8(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const int8_t* wg,
                      const float* sg, const int8_t* wu, const float* su, int64_t N, int epi,
                      void* out, int64_t ldo, int8_t* out_q, float* out_s, cudaStream_t st) {
  if (int r = check_common(a_q, a_s, M, K, N)) return r;
  if (int r = check_n(N)) return r;
  if (M == 0 || N == 0) return QLIN_OK;
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = seg_w8(a.seg[0], wg, sg, K, N)) return r;
  if (int r = seg_w8(a.seg[1], wu, su, K, N)) return r;
  a.nseg = 2;
  a.a_q = a_q;
  a.a_s = a_s;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = 64;
  a.out = out;
  a.ldo = ldo;
  a.out_q = out_q;
  a.out_s = out_s;
  a.n_q = static_cast<int>(N);
  return run_gemv(8, epi, a, tiles_of(N), st);
}

int qlin_mlp_gate_up(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const int8_t* wg,
                     const float* sg, const int8_t* wu, const float* su, int64_t N, void* out,
                     int64_t ldo, void* stream) {
  if (M > 0 && N > 0 && !out) return fail(QLIN_ERR_INVALID_ARGUMENT, "null out");
  if (ldo < N) return fail(QLIN_ERR_SHAPE, "row stride smaller than N");
  return gate_up_w8(a_q, a_s, M, K, wg, sg, wu, su, N, kEpiSiluBf16, out, ldo, nullptr, nullptr,
                    static_cast<cudaStream_t>(stream));
}

int qlin_mlp_gate_up_quant(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                           const int8_t* wg, const float* sg, const int8_t* wu, const float* su,
                           int64_t N, int8_t* out_q, float* out_s, void* stream) {
  if (N % 64 != 0) return fail(QLIN_ERR_SHAPE, "N=%lld must be a multiple of 64", (long long)N);
  if (M > 0 && N > 0 && (!out_q || !out_s)) return fail(QLIN_ERR_INVALID_ARGUMENT, "null output");
  return gate_up_w8(a_q, a_s, M, K, wg, sg, wu, su, N, kEpiSiluQuant, nullptr, 0, out_q, out_s,
                    static_cast<cudaStream_t>(stream));
}

int qlin_mlp_gate_up_quant_w4(const int8_t* a_q, const float* a_s, int64_t M, int64_t K,
                              const uint8_t* wg, const void* sg, const uint8_t* zg, const uint8_t* wu,
                              const void* su, const uint8_t* zu, int64_t N, int64_t wgrp,
                              int8_t* out_q, float* out_s, void* stream) {
  if (int r = check_common(a_q, a_s, M, K, N)) return r;
  if (int r = check_n(N)) return r;
  if (int r = check_wgrp(K, wgrp)) return r;
  if (N % 64 != 0) return fail(QLIN_ERR_SHAPE, "N=%lld must be a multiple of 64", (long long)N);
  if (M == 0 || N == 0) return QLIN_OK;
  if (!out_q || !out_s) return fail(QLIN_ERR_INVALID_ARGUMENT, "null output");
  GemvArgs a;
  memset(&a, 0, sizeof(a));
  if (int r = seg_w4(a.seg[0], wg, sg, zg, K, N, wgrp)) return r;
  if (int r = seg_w4(a.seg[1], wu, su, zu, K, N, wgrp)) return r;
  a.nseg = 2;
  a.a_q = a_q;
  a.a_s = a_s;
  a.M = static_cast<int>(M);
  a.K = static_cast<int>(K);
  a.wgrp = static_cast<int>(wgrp);
  a.out_q = out_q;
  a.out_s = out_s;
  a.n_q = static_cast<int>(N);
  return run_gemv(4, kEpiSiluQuant, a, tiles_of(N), static_cast<cudaStream_t>(stream));
}

int qlin_quant_row(const void* x, int64_t ldx, int64_t M, int64_t K, int8_t* q, float* s,
                   void* stream) {
  if (M < 0 || K < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "negative size");
  if (K == 0 || K % kGroup != 0) return fail(QLIN_ERR_SHAPE, "K=%lld must be a positive multiple of 64", (long long)K);
  if (M == 0) return QLIN_OK;
  if (M > 65535) return fail(QLIN_ERR_SHAPE, "M=%lld too large", (long long)M);
  if (!x || !q || !s) return fail(QLIN_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldx < K) return fail(QLIN_ERR_SHAPE, "row stride smaller than K");
  if (!aligned(x, 4) || (ldx % 2) != 0 || !aligned(q, 2) || !aligned(s, 4))
    return fail(QLIN_ERR_ALIGNMENT, "x needs 4-byte aligned rows, q 2-byte, s 4-byte alignment");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  const int G = static_cast<int>(K / kGroup);
  // 16-byte rows: 8 elements per lane (measured on B200 at M = K = 2048: ~10 us
  // with 2 elements per lane); otherwise the 2-element kernel.
  const bool vec = aligned(x, 16) && ldx % 8 == 0 && aligned(q, 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = vec ? dim3((G + kQuantVecGroups - 1) / kQuantVecGroups, static_cast<unsigned>(M), 1)
                    : dim3((G + kQuantWarps - 1) / kQuantWarps, static_cast<unsigned>(M), 1);
  cfg.blockDim = dim3(kQuantWarps * 32, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (int r = prefer_shared(vec ? reinterpret_cast<const void*>(quant_row_vec_kernel)
                                : reinterpret_cast<const void*>(quant_row_kernel)))
    return r;
  cudaError_t e = cudaLaunchKernelEx(&cfg, vec ? quant_row_vec_kernel : quant_row_kernel,
                                     static_cast<const __nv_bfloat16*>(x),
                                     static_cast<long long>(ldx), static_cast<int>(M),
                                     static_cast<int>(K), q, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(quant_row)");
  return QLIN_OK;
}


int qlin_rmsnorm_quant(const void* x, int64_t ldx, const void* w, int64_t M, int64_t K, float eps, int one_plus,
                       int8_t* q, float* s, void* stream) {
  if (int r = check_rows(M, K, "rmsnorm_quant")) return r;
  if (K == 0 || K % kGroup != 0 || K > 16384)
    return fail(QLIN_ERR_SHAPE, "rmsnorm_quant: K=%lld must be a positive multiple of 64, at most 16384", (long long)K);
  if (M == 0) return QLIN_OK;
  if (M > 2147483647) return fail(QLIN_ERR_SHAPE, "rmsnorm_quant: M too large");
  if (!x || !w || !q || !s) return fail(QLIN_ERR_INVALID_ARGUMENT, "rmsnorm_quant: null pointer");
  if (ldx < K) return fail(QLIN_ERR_SHAPE, "rmsnorm_quant: row stride smaller than K");
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(w, 16) || !aligned(q, 8) || !aligned(s, 4))
    return fail(QLIN_ERR_ALIGNMENT, "rmsnorm_quant: x and w need 16-byte aligned rows, q 8-byte, s 4-byte alignment");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  const int nch = static_cast<int>(K / 8);
  const int nv = (nch + kProdThreads - 1) / kProdThreads;
  long long ldx_ = ldx;
  int K_ = static_cast<int>(K), one_plus_ = one_plus ? 1 : 0;
  float eps_ = eps;
  void* args[] = {const_cast<void**>(&x), &ldx_, const_cast<void**>(&w), &K_, &eps_, &one_plus_, &q, &s};
  const void* kern = nv <= 1   ? reinterpret_cast<const void*>(rmsnorm_quant_kernel<1>)
                     : nv <= 2 ? reinterpret_cast<const void*>(rmsnorm_quant_kernel<2>)
                     : nv <= 4 ? reinterpret_cast<const void*>(rmsnorm_quant_kernel<4>)
                               : reinterpret_cast<const void*>(rmsnorm_quant_kernel<8>);
  return prod_launch(kern, dim3(static_cast<unsigned>(M)), args, static_cast<cudaStream_t>(stream));
}

static int norm_gated_common(const void* v, const void* z, int64_t ldz, const void* w, int64_t T, int64_t N,
                             int64_t HD, float eps, int8_t* q, float* s, void* out, void* stream) {
  const bool quant = out == nullptr;
  if (int r = check_rows(T, N, "norm_gated")) return r;
  if (!(HD == 64 || HD == 128 || HD == 256) || N % HD != 0)
    return fail(QLIN_ERR_SHAPE, "norm_gated: head dim %lld must be 64, 128 or 256 and divide N=%lld", (long long)HD,
                (long long)N);
  if (T == 0 || N == 0) return QLIN_OK;
  if (!v || !z || !w || (quant && (!q || !s))) return fail(QLIN_ERR_INVALID_ARGUMENT, "norm_gated: null pointer");
  if (ldz < N) return fail(QLIN_ERR_SHAPE, "norm_gated: z row stride smaller than N");
  if (!aligned(v, 4) || !aligned(z, 4) || ldz % 2 != 0 || !aligned(w, 4) || (quant && !aligned(s, 4)))
    return fail(QLIN_ERR_ALIGNMENT, "norm_gated: v, z rows and w need 4-byte alignment");
  const long long items = T * (N / HD);
  if (items > 65535ll * 65535 * 8) return fail(QLIN_ERR_SHAPE, "norm_gated: too many heads");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  long long ldz_ = ldz;
  int T_ = static_cast<int>(T), NV = static_cast<int>(N / HD);
  float eps_ = eps;
  void* args[] = {const_cast<void**>(&v), const_cast<void**>(&z), &ldz_, const_cast<void**>(&w), &T_, &NV, &eps_,
                  &q, &s, &out};
  const void* kern;
  if (quant) {
    kern = HD == 64    ? reinterpret_cast<const void*>(norm_gated_kernel<64, true>)
           : HD == 128 ? reinterpret_cast<const void*>(norm_gated_kernel<128, true>)
                       : reinterpret_cast<const void*>(norm_gated_kernel<256, true>);
  } else {
    kern = HD == 64    ? reinterpret_cast<const void*>(norm_gated_kernel<64, false>)
           : HD == 128 ? reinterpret_cast<const void*>(norm_gated_kernel<128, false>)
                       : reinterpret_cast<const void*>(norm_gated_kernel<256, false>);
  }
  const unsigned blocks = static_cast<unsigned>((items + kProdThreads / 32 - 1) / (kProdThreads / 32));
  return prod_launch(kern, dim3(blocks), args, static_cast<cudaStream_t>(stream));
}

int qlin_norm_gated_quant(const void* v, const void* z, int64_t ldz, const void* w, int64_t T, int64_t N, int64_t HD,
                          float eps, int8_t* q, float* s, void* stream) {
  if (!q || !s) return fail(QLIN_ERR_INVALID_ARGUMENT, "norm_gated_quant: null output");
  return norm_gated_common(v, z, ldz, w, T, N, HD, eps, q, s, nullptr, stream);
}

int qlin_norm_gated(const void* v, const void* z, int64_t ldz, const void* w, int64_t T, int64_t N, int64_t HD,
                    float eps, void* out, void* stream) {
  if (!out) return fail(QLIN_ERR_INVALID_ARGUMENT, "norm_gated: null output");
  return norm_gated_common(v, z, ldz, w, T, N, HD, eps, nullptr, nullptr, out, stream);
}

static int mul_quant_common(bool gate_mul, const void* a, int64_t lda, const void* g, int64_t ldg, int64_t M,
                            int64_t N, int64_t HD, int8_t* q, float* s, void* stream) {
  const char* what = gate_mul ? "gate_mul_quant" : "silu_mul_quant";
  if (int r = check_rows(M, N, what)) return r;
  if (N % kGroup != 0) return fail(QLIN_ERR_SHAPE, "%s: N=%lld must be a multiple of 64", what, (long long)N);
  if (gate_mul && (HD <= 0 || HD % 8 != 0 || N % HD != 0))
    return fail(QLIN_ERR_SHAPE, "%s: head dim %lld must be a multiple of 8 dividing N", what, (long long)HD);
  if (M == 0 || N == 0) return QLIN_OK;
  if (M > 65535) return fail(QLIN_ERR_SHAPE, "%s: M=%lld too large", what, (long long)M);
  if (!a || !g || !q || !s) return fail(QLIN_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  const int64_t gcols = gate_mul ? 2 * N : N;
  if (lda < N || ldg < gcols) return fail(QLIN_ERR_SHAPE, "%s: row stride too small", what);
  if (!aligned(a, 16) || !aligned(g, 16) || lda % 8 != 0 || ldg % 8 != 0 || !aligned(q, 8) || !aligned(s, 4))
    return fail(QLIN_ERR_ALIGNMENT, "%s: inputs need 16-byte aligned rows, q 8-byte, s 4-byte alignment", what);
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  long long lda_ = lda, ldg_ = ldg;
  int N_ = static_cast<int>(N), HD_ = static_cast<int>(gate_mul ? HD : 8);
  void* args[] = {const_cast<void**>(&a), &lda_, const_cast<void**>(&g), &ldg_, &N_, &HD_, &q, &s};
  const void* kern = gate_mul ? reinterpret_cast<const void*>(mul_quant_kernel<true>)
                              : reinterpret_cast<const void*>(mul_quant_kernel<false>);
  const unsigned cblocks = static_cast<unsigned>((N / 8 + kProdThreads - 1) / kProdThreads);
  return prod_launch(kern, dim3(cblocks, static_cast<unsigned>(M)), args, static_cast<cudaStream_t>(stream));
}

int qlin_gate_mul_quant(const void* a, const void* g, int64_t ldg, int64_t M, int64_t N, int64_t hd, int8_t* q,
                        float* s, void* stream) {
  return mul_quant_common(true, a, N, g, ldg, M, N, hd, q, s, stream);
}

int qlin_silu_mul_quant(const void* g, const void* u, int64_t M, int64_t N, int8_t* q, float* s, void* stream) {
  // y = silu(g) * u: the kernel's first operand is the multiplier (u), the second the activation input (g)
  return mul_quant_common(false, u, N, g, N, M, N, 0, q, s, stream);
}

int qlin_gate_proj(const int8_t* a_q, const float* a_s, int64_t M, int64_t K, const void* wb, const void* wa,
                   int64_t NB, const void* dt_bias, const void* a_log, float* beta, float* gate, void* stream) {
  if (int r = check_rows(M, K, "gate_proj")) return r;
  if (K == 0 || K % kGroup != 0) return fail(QLIN_ERR_SHAPE, "gate_proj: K=%lld must be a positive multiple of 64", (long long)K);
  if (NB < 1 || NB > 65535) return fail(QLIN_ERR_SHAPE, "gate_proj: NB=%lld out of range", (long long)NB);
  if (M == 0) return QLIN_OK;
  if (M > 2147483647) return fail(QLIN_ERR_SHAPE, "gate_proj: M too large");
  if (!a_q || !a_s || !wb || !wa || !dt_bias || !a_log || !beta || !gate)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "gate_proj: null pointer");
  if (!aligned(a_q, 8) || !aligned(wb, 16) || !aligned(wa, 16) || !aligned(a_s, 4) || !aligned(beta, 4) ||
      !aligned(gate, 4) || !aligned(dt_bias, 2) || !aligned(a_log, 2))
    return fail(QLIN_ERR_ALIGNMENT, "gate_proj: a_q 8-byte, wb/wa 16-byte aligned");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  int K_ = static_cast<int>(K), NB_ = static_cast<int>(NB);
  void* args[] = {const_cast<int8_t**>(&a_q), const_cast<float**>(&a_s), &K_, const_cast<void**>(&wb),
                  const_cast<void**>(&wa), &NB_, const_cast<void**>(&dt_bias), const_cast<void**>(&a_log), &beta,
                  &gate};
  if (M > 65535) return fail(QLIN_ERR_SHAPE, "gate_proj: M=%lld too large", (long long)M);
  return prod_launch(reinterpret_cast<const void*>(gate_proj_kernel),
                     dim3(static_cast<unsigned>(NB), static_cast<unsigned>(M)), args, static_cast<cudaStream_t>(stream));
}


int qlin_qk_norm_rope(const void* proj, int64_t ldp, const void* qn, const void* kn, const float* invf, int64_t rd,
                      void* qout, void* kvc, float* kvs, int64_t T, int64_t nq, int64_t nkv, int64_t hd, int64_t pos0,
                      const int32_t* pos_dev, float eps, int kv_int8, int batch, int64_t kv_stride,
                      int64_t kvs_stride, void* stream) {
  if (T < 0 || nq <= 0 || nkv <= 0 || pos0 < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "qk_norm_rope: bad size");
  if (!(hd == 128 || hd == 256)) return fail(QLIN_ERR_SHAPE, "qk_norm_rope: head dim %lld (128 or 256)", (long long)hd);
  const int E = static_cast<int>(hd / 32);
  if (rd <= 0 || rd > hd || rd % (2 * E) != 0 || ((rd / 2) / E) > 16)
    return fail(QLIN_ERR_SHAPE, "qk_norm_rope: rotary dims %lld must be a multiple of %d up to head dim", (long long)rd,
                2 * E);
  if (T == 0) return QLIN_OK;
  if (!proj || !qn || !kn || !invf || !qout || !kvc || (kv_int8 && !kvs))
    return fail(QLIN_ERR_INVALID_ARGUMENT, "qk_norm_rope: null pointer");
  if (ldp < (2 * nq + 2 * nkv) * hd) return fail(QLIN_ERR_SHAPE, "qk_norm_rope: projection row too short");
  if (!aligned(proj, 16) || ldp % 8 != 0 || !aligned(qn, 16) || !aligned(kn, 16) || !aligned(qout, 16) ||
      !aligned(kvc, 16) || !aligned(invf, 4) || (kvs && !aligned(kvs, 4)) || (pos_dev && !aligned(pos_dev, 4)))
    return fail(QLIN_ERR_ALIGNMENT, "qk_norm_rope: 16-byte aligned rows required");
  if (batch && (kv_stride < 0 || kvs_stride < 0)) return fail(QLIN_ERR_INVALID_ARGUMENT, "qk_norm_rope: strides");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  QkRopeArgs a;
  a.proj = static_cast<const __nv_bfloat16*>(proj);
  a.ldp = ldp;
  a.qn = static_cast<const __nv_bfloat16*>(qn);
  a.kn = static_cast<const __nv_bfloat16*>(kn);
  a.invf = invf;
  a.qout = static_cast<__nv_bfloat16*>(qout);
  a.kvc = kvc;
  a.kvs = kvs;
  a.pos_dev = pos_dev;
  a.kv_stride = batch ? kv_stride : 0;
  a.kvs_stride = batch ? kvs_stride : 0;
  a.T = static_cast<int>(T);
  a.nq = static_cast<int>(nq);
  a.nkv = static_cast<int>(nkv);
  a.rd = static_cast<int>(rd);
  a.pos0 = static_cast<int>(pos0);
  a.batch = batch ? 1 : 0;
  a.eps = eps;
  const long long warps = T * (nq + 2 * nkv);
  const unsigned blocks = static_cast<unsigned>((warps + kDecThreads / 32 - 1) / (kDecThreads / 32));
  const void* kern = hd == 256 ? (kv_int8 ? reinterpret_cast<const void*>(qk_norm_rope_kernel<256, true>)
                                          : reinterpret_cast<const void*>(qk_norm_rope_kernel<256, false>))
                               : (kv_int8 ? reinterpret_cast<const void*>(qk_norm_rope_kernel<128, true>)
                                          : reinterpret_cast<const void*>(qk_norm_rope_kernel<128, false>));
  void* args[] = {&a};
  return dec_launch(kern, dim3(blocks), dim3(kDecThreads), 0, 1, args, static_cast<cudaStream_t>(stream));
}

int qlin_attn_decode(const void* q, const void* kvc, const float* kvs, void* out, int64_t pos, const int32_t* pos_dev,
                     int64_t max_pos, int64_t batch, int64_t nq, int64_t nkv, int64_t hd, int kv_int8,
                     int64_t kv_stride, int64_t kvs_stride, void* stream) {
  if (batch <= 0 || nq <= 0 || nkv <= 0 || nq % nkv != 0 || pos < 0)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "attn_decode: bad size");
  if (!(hd == 128 || hd == 256)) return fail(QLIN_ERR_SHAPE, "attn_decode: head dim %lld (128 or 256)", (long long)hd);
  if (batch > 65535 || nkv > 65535) return fail(QLIN_ERR_SHAPE, "attn_decode: too many candidates / heads");
  if (!q || !kvc || !out || (kv_int8 && !kvs)) return fail(QLIN_ERR_INVALID_ARGUMENT, "attn_decode: null pointer");
  if (!aligned(q, 16) || !aligned(kvc, 16) || (kvs && !aligned(kvs, 4)) || (pos_dev && !aligned(pos_dev, 4)))
    return fail(QLIN_ERR_ALIGNMENT, "attn_decode: q and the cache need 16-byte alignment");
  if (batch > 1 && (kv_stride <= 0 || (kv_int8 && kvs_stride <= 0)))
    return fail(QLIN_ERR_INVALID_ARGUMENT, "attn_decode: per-candidate cache strides required for batch > 1");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  AttnDecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kvc = kvc;
  a.kvs = kvs;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.pos_dev = pos_dev;
  a.kv_stride = batch > 1 ? kv_stride : 0;
  a.kvs_stride = batch > 1 ? kvs_stride : 0;
  a.pos = static_cast<int>(pos);
  a.nq = static_cast<int>(nq);
  a.nkv = static_cast<int>(nkv);
  // positions per CTA: about 64 (8 warps x 8), clusters of up to 8 CTAs; with
  // a device-side position the split follows the largest position expected
  const long long n = (pos_dev ? (max_pos > pos ? max_pos : pos) : pos) + 1;
  int S = static_cast<int>((n + 63) / 64);
  if (S > tune_ad_smax()) S = tune_ad_smax();
  if (S < 1) S = 1;
  const int Gfull = static_cast<int>(nq / nkv);
  if (!(Gfull == 1 || Gfull == 2 || Gfull == 4 || Gfull == 8))
    return fail(QLIN_ERR_SHAPE, "attn_decode: %d query heads per KV head (1, 2, 4 or 8)", Gfull);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int B = static_cast<int>(batch), NKV = static_cast<int>(nkv);
  // Split a KV head's query heads over more CTAs until the launch covers the
  // SMs (the extra reads of the same cache rows mostly hit L2).  Measured on
  // B200, config 4 (B = 4, 8 query / 2 KV heads, 1025 int8 positions, graph
  // replay): 12.9 us with the heads split over 4 CTA groups (256 CTAs in
  // clusters of 8), 22.6 us over 2, 19.1 us unsplit; clusters of 4 at the
  // 4-way split 18.7 us.
  int hsplit = 1;
  while (hsplit < Gfull && static_cast<long long>(S) * NKV * hsplit * B < di.sms) hsplit *= 2;
  if (tune_ad_hsplit() > 0 && tune_ad_hsplit() <= Gfull && Gfull % tune_ad_hsplit() == 0) hsplit = tune_ad_hsplit();
  if (static_cast<long long>(NKV) * hsplit > 65535) hsplit = 1;
  a.hsplit = hsplit;
  const int G = Gfull / hsplit;
  if (hd == 256)
    return kv_int8 ? attn_decode_g<8, true>(G, a, S, NKV * hsplit, B, st)
                   : attn_decode_g<8, false>(G, a, S, NKV * hsplit, B, st);
  return kv_int8 ? attn_decode_g<4, true>(G, a, S, NKV * hsplit, B, st)
                 : attn_decode_g<4, false>(G, a, S, NKV * hsplit, B, st);
}

int qlin_delta_decode(const void* qkv, int64_t ldq, const float* g, const float* beta, float* state, void* out,
                      int64_t batch, int64_t nh, int64_t dk, int64_t dv, void* stream) {
  if (batch <= 0 || nh <= 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "delta_decode: bad size");
  if (dk != kDeltaDK || dv != kDeltaDV) return fail(QLIN_ERR_SHAPE, "delta_decode: head dims must be 128 x 128");
  if (batch > 65535 || nh > 65535) return fail(QLIN_ERR_SHAPE, "delta_decode: too many candidates / heads");
  if (!qkv || !g || !beta || !state || !out) return fail(QLIN_ERR_INVALID_ARGUMENT, "delta_decode: null pointer");
  if (batch > 1 && ldq < (2 * dk + dv) * nh) return fail(QLIN_ERR_SHAPE, "delta_decode: qkv row stride too small");
  if (!aligned(qkv, 2) || !aligned(state, 16) || !aligned(out, 2) || !aligned(g, 4) || !aligned(beta, 4))
    return fail(QLIN_ERR_ALIGNMENT, "delta_decode: state needs 16-byte alignment");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  long long ldq_ = batch > 1 ? ldq : 0;
  int nh_ = static_cast<int>(nh);
  const __nv_bfloat16* qp = static_cast<const __nv_bfloat16*>(qkv);
  __nv_bfloat16* op = static_cast<__nv_bfloat16*>(out);
  void* args[] = {&qp, &ldq_, const_cast<float**>(&g), const_cast<float**>(&beta), &state, &op, &nh_};
  return dec_launch(reinterpret_cast<const void*>(delta_decode_kernel),
                    dim3(static_cast<unsigned>(nh), static_cast<unsigned>(batch), kDeltaDV / 32),
                    dim3(kDeltaWarps * 32), 0, 1, args, static_cast<cudaStream_t>(stream));
}

int qlin_conv_silu(const void* x, int64_t ldx, const void* w, int64_t ks, const void* state, void* y, int64_t T,
                   int64_t C, int batch, void* stream) {
  if (T < 0 || C < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "conv_silu: bad size");
  if (ks != kConvKS) return fail(QLIN_ERR_SHAPE, "conv_silu: kernel width %lld (4 supported)", (long long)ks);
  if (C % 8 != 0) return fail(QLIN_ERR_SHAPE, "conv_silu: channels must be a multiple of 8");
  if (T == 0 || C == 0) return QLIN_OK;
  if (T > 65535) return fail(QLIN_ERR_SHAPE, "conv_silu: T too large");
  if (!x || !w || !state || !y) return fail(QLIN_ERR_INVALID_ARGUMENT, "conv_silu: null pointer");
  if (ldx < C) return fail(QLIN_ERR_SHAPE, "conv_silu: row stride smaller than C");
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(w, 16) || !aligned(state, 16) || !aligned(y, 16))
    return fail(QLIN_ERR_ALIGNMENT, "conv_silu: 16-byte aligned rows required");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  long long ldx_ = ldx;
  int T_ = static_cast<int>(T), C_ = static_cast<int>(C), b_ = batch ? 1 : 0;
  void* args[] = {const_cast<void**>(&x), &ldx_, const_cast<void**>(&w), const_cast<void**>(&state), &y, &T_, &C_, &b_};
  const unsigned cb = static_cast<unsigned>((C / 8 + kDecThreads - 1) / kDecThreads);
  return dec_launch(reinterpret_cast<const void*>(conv_silu_kernel), dim3(cb, static_cast<unsigned>(T)),
                    dim3(kDecThreads), 0, 1, args, static_cast<cudaStream_t>(stream));
}

int qlin_conv_state_update(const void* x, int64_t ldx, void* state, int64_t T, int64_t C, int64_t ks, int64_t batch,
                           void* stream) {
  if (T < 0 || C < 0 || batch <= 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "conv_state_update: bad size");
  if (ks != kConvKS) return fail(QLIN_ERR_SHAPE, "conv_state_update: kernel width %lld (4 supported)", (long long)ks);
  if (C % 8 != 0) return fail(QLIN_ERR_SHAPE, "conv_state_update: channels must be a multiple of 8");
  if (T == 0 || C == 0) return QLIN_OK;
  if (batch > 1 && batch != T) return fail(QLIN_ERR_SHAPE, "conv_state_update: batch mode takes one row per candidate");
  if (batch > 65535) return fail(QLIN_ERR_SHAPE, "conv_state_update: batch too large");
  if (!x || !state) return fail(QLIN_ERR_INVALID_ARGUMENT, "conv_state_update: null pointer");
  if (ldx < C) return fail(QLIN_ERR_SHAPE, "conv_state_update: row stride smaller than C");
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(state, 16))
    return fail(QLIN_ERR_ALIGNMENT, "conv_state_update: 16-byte aligned rows required");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  long long ldx_ = ldx;
  int T_ = static_cast<int>(T), C_ = static_cast<int>(C), b_ = batch > 1 ? 1 : 0;
  void* args[] = {const_cast<void**>(&x), &ldx_, &state, &T_, &C_, &b_};
  const unsigned cb = static_cast<unsigned>((C / 8 + kDecThreads - 1) / kDecThreads);
  return dec_launch(reinterpret_cast<const void*>(conv_state_update_kernel),
                    dim3(cb, static_cast<unsigned>(batch > 1 ? batch : 1)), dim3(kDecThreads), 0, 1, args,
                    static_cast<cudaStream_t>(stream));
}

int qlin_conv_silu_update(const void* x, int64_t ldx, const void* w, int64_t ks, void* state, void* y, int64_t batch,
                          int64_t C, void* stream) {
  if (batch < 0 || C < 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "conv_silu_update: bad size");
  if (ks != kConvKS) return fail(QLIN_ERR_SHAPE, "conv_silu_update: kernel width %lld (4 supported)", (long long)ks);
  if (C % 8 != 0) return fail(QLIN_ERR_SHAPE, "conv_silu_update: channels must be a multiple of 8");
  if (batch == 0 || C == 0) return QLIN_OK;
  if (batch > 65535) return fail(QLIN_ERR_SHAPE, "conv_silu_update: batch too large");
  if (!x || !w || !state || !y) return fail(QLIN_ERR_INVALID_ARGUMENT, "conv_silu_update: null pointer");
  if (ldx < C) return fail(QLIN_ERR_SHAPE, "conv_silu_update: row stride smaller than C");
  if (!aligned(x, 16) || ldx % 8 != 0 || !aligned(w, 16) || !aligned(state, 16) || !aligned(y, 16))
    return fail(QLIN_ERR_ALIGNMENT, "conv_silu_update: 16-byte aligned rows required");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  long long ldx_ = ldx;
  int C_ = static_cast<int>(C);
  void* args[] = {const_cast<void**>(&x), &ldx_, const_cast<void**>(&w), &state, &y, &C_};
  const unsigned cb = static_cast<unsigned>((C / 8 + kDecThreads - 1) / kDecThreads);
  return dec_launch(reinterpret_cast<const void*>(conv_silu_update_kernel), dim3(cb, static_cast<unsigned>(batch)),
                    dim3(kDecThreads), 0, 1, args, static_cast<cudaStream_t>(stream));
}


int qlin_attn_prefill(const void* q, const void* kvc, const float* kvs, void* out, int64_t T, int64_t pos0,
                      int64_t nq, int64_t nkv, int64_t hd, int kv_int8, void* stream) {
  if (T < 0 || pos0 < 0 || nq <= 0 || nkv <= 0 || nq % nkv != 0)
    return fail(QLIN_ERR_INVALID_ARGUMENT, "attn_prefill: bad size");
  if (!(hd == 128 || hd == 256)) return fail(QLIN_ERR_SHAPE, "attn_prefill: head dim %lld (128 or 256)", (long long)hd);
  if (T == 0) return QLIN_OK;
  if (nq > 65535 || (T + kPaRows - 1) / kPaRows > 2147483647ll || pos0 + T > 2147483647ll)
    return fail(QLIN_ERR_SHAPE, "attn_prefill: too large");
  if (!q || !kvc || !out || (kv_int8 && !kvs)) return fail(QLIN_ERR_INVALID_ARGUMENT, "attn_prefill: null pointer");
  if (!aligned(q, 16) || !aligned(kvc, 16) || !aligned(out, 4) || (kvs && !aligned(kvs, 4)))
    return fail(QLIN_ERR_ALIGNMENT, "attn_prefill: q and the cache need 16-byte alignment");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  AttnPrefillArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kvc = kvc;
  a.kvs = kvs;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.T = static_cast<int>(T);
  a.pos0 = static_cast<int>(pos0);
  a.nq = static_cast<int>(nq);
  a.nkv = static_cast<int>(nkv);
  const void* kern = hd == 256 ? (kv_int8 ? reinterpret_cast<const void*>(attn_prefill_kernel<256, true>)
                                          : reinterpret_cast<const void*>(attn_prefill_kernel<256, false>))
                               : (kv_int8 ? reinterpret_cast<const void*>(attn_prefill_kernel<128, true>)
                                          : reinterpret_cast<const void*>(attn_prefill_kernel<128, false>));
  const size_t smem = attn_prefill_smem(static_cast<int>(hd));
  static std::atomic<unsigned long long> done[4];  // one opt-in per kernel instance and device
  const int inst = (hd == 256 ? 2 : 0) + (kv_int8 ? 1 : 0);
  if (int r = smem_optin(kern, smem, done[inst])) return r;
  void* args[] = {&a};
  return dec_launch(kern, dim3(static_cast<unsigned>((T + kPaRows - 1) / kPaRows), static_cast<unsigned>(nq)),
                    dim3(kPaThreads), smem, 1, args, static_cast<cudaStream_t>(stream));
}

int qlin_delta_prefill(const void* qkv, int64_t ldq, const float* g, const float* beta, float* state, void* out,
                       int64_t T, int64_t nh, int64_t dk, int64_t dv, void* stream) {
  if (T < 0 || nh <= 0) return fail(QLIN_ERR_INVALID_ARGUMENT, "delta_prefill: bad size");
  if (dk != kDpDK || dv % kDpVS != 0 || dv <= 0)
    return fail(QLIN_ERR_SHAPE, "delta_prefill: key dim must be 128 and the value dim a multiple of 32");
  if (T == 0) return QLIN_OK;
  if (T > 2147483647ll || nh > 65535) return fail(QLIN_ERR_SHAPE, "delta_prefill: too large");
  if (!qkv || !g || !beta || !state || !out) return fail(QLIN_ERR_INVALID_ARGUMENT, "delta_prefill: null pointer");
  if (ldq < (2 * dk + dv) * nh) return fail(QLIN_ERR_SHAPE, "delta_prefill: qkv row stride too small");
  if (!aligned(qkv, 16) || ldq % 8 != 0 || !aligned(state, 4) || !aligned(out, 2) || !aligned(g, 4) ||
      !aligned(beta, 4))
    return fail(QLIN_ERR_ALIGNMENT, "delta_prefill: qkv needs 16-byte aligned rows");
  DevInfo di;
  if (int r = launch_info(&di)) return r;
  DeltaPrefillArgs a;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldq = ldq;
  a.g = g;
  a.beta = beta;
  a.state = state;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.T = static_cast<int>(T);
  a.nh = static_cast<int>(nh);
  a.dv = static_cast<int>(dv);
  static std::atomic<unsigned long long> done{0};
  const void* kern = reinterpret_cast<const void*>(delta_prefill_kernel);
  if (int r = smem_optin(kern, sizeof(DpSmem), done)) return r;
  void* args[] = {&a};
  return dec_launch(kern, dim3(static_cast<unsigned>(nh), static_cast<unsigned>(dv / kDpVS)), dim3(kDpThreads),
                    sizeof(DpSmem), 1, args, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
