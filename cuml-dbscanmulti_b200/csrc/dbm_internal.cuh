// dbm_internal.cuh -- shared device helpers and host plumbing of libdbm.so (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/dbm.h"

namespace dbm {

// ---- status plumbing (host) ------------------------------------------------------------
struct Status {
  int code = DBM_OK;
  std::string msg;
  bool ok() const { return code == DBM_OK; }
  static Status Ok() { return Status{}; }
  static Status Err(int c, std::string m) { return Status{c, std::move(m)}; }
};

#define DBM_CUDA(call)                                                                       \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      return ::dbm::Status::Err(e_ == cudaErrorMemoryAllocation ? DBM_ERR_OOM : DBM_ERR_CUDA, \
                                std::string(#call) + ": " + cudaGetErrorString(e_));         \
  } while (0)

#define DBM_TRY(expr)                 \
  do {                                \
    ::dbm::Status s_ = (expr);        \
    if (!s_.ok()) return s_;          \
  } while (0)

// ---- constants -------------------------------------------------------------------------
constexpr uint8_t kNoNeighbor = 255;      // per-pair code when no eps contains the pair
constexpr int kMaxEps = DBM_MAX_EPS;
constexpr uint32_t kColMask = 0x0FFFFFFFu; // packed neighbour word: code << 28 | column
constexpr int kCodeShift = 28;
constexpr int32_t kNone = INT32_MAX;       // "no label yet" / noise before relabel

// device error flags (bitmask written by kernels, read by the host after a stage)
constexpr int kErrTmaTimeout = 1;
constexpr int kErrUnionLimit = 2;
constexpr int kErrNonFinite = 4;
constexpr int kErrGraphMismatch = 8;  // a batch's re-derived pairs disagree with the degree pass

// ---- small device helpers ----------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// mbarrier / TMA (PTX ISA 8.x, sm_90+; used here on sm_100a)
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init()
{
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
  uint32_t done;
  asm volatile(
    "{\n\t.reg .pred p;\n\t"
    "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
    "selp.u32 %0, 1, 0, p;\n\t}"
    : "=r"(done)
    : "r"(smem_u32(bar)), "r"(parity)
    : "memory");
  return done != 0;
}
// Bounded wait: gives up after `limit` polls (each poll may suspend briefly in hardware).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit)
{
  for (uint32_t it = 0; it < limit; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void fence_proxy_async_smem()
{
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 2-D tiled TMA load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint64_t* bar)
{
  asm volatile(
    "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
    " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
    "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
    : "memory");
}

// ---- a shard's share of the distance work items ----------------------------------------------
// Runs of kShardRun consecutive items are dealt round-robin over the S shards (run r to shard
// r % S): the ranks' shares cost alike whatever the cost profile along the J-major worklist
// (contiguous thirds or halves did not: the dense parts of the point set land on one rank),
// while each run keeps the worklist's locality (consecutive items of one tile J).  Local item i
// of shard s is global item shard_item(i, s, S); the shard's valid local items are a prefix.
constexpr int64_t kShardRun = 64;
__host__ __device__ __forceinline__ int64_t shard_item(int64_t i, int s, int S)
{
  return ((i / kShardRun) * S + s) * kShardRun + i % kShardRun;
}
__host__ __device__ __forceinline__ int64_t shard_items(int64_t total, int s, int S)
{
  const int64_t runs = (total + kShardRun - 1) / kShardRun;
  if (s >= runs) return 0;
  const int64_t mine = (runs - 1 - s) / S + 1;
  const int64_t last = s + (mine - 1) * S;  // global index of this shard's last run
  return mine * kShardRun - (last == runs - 1 ? runs * kShardRun - total : 0);
}

// ---- union-find with minimum-index roots --------------------------------------------------
// Roots are always the smallest index of their tree: a root is only ever re-pointed at a
// smaller root, so a fully compressed parent array maps every member to its component's
// minimum index.  Path splitting (each visited node is re-pointed at its grandparent) writes only
// ancestors, so concurrent finds are safe; one dependent load per step: the grandparent read for
// the split is the next step's parent (a value another thread has moved on since is still an
// ancestor, so the walk still ends at a root as read).  The parent of x is parent[x * stride]
// (forests of several configs interleaved point by point).
__device__ __forceinline__ int32_t uf_find(int32_t* parent, int32_t x, int stride = 1)
{
  volatile int32_t* p = parent;
  int32_t px = p[static_cast<int64_t>(x) * stride];
  while (px != x) {
    const int32_t gp = p[static_cast<int64_t>(px) * stride];
    if (gp != px) p[static_cast<int64_t>(x) * stride] = gp;
    x = px;
    px = gp;
  }
  return x;
}

// Neighbour entries per batch row from which a batch's labelling takes the sampled union path
// (and needs the root snapshot, kSnapBytesPerPoint per eps and point).
constexpr int64_t kDenseEntriesPerRow = 64;
constexpr int64_t kSnapBytesPerPoint = 32;

// Retry bound of uf_unite: a hook can lose its CAS to a concurrent hook at most once per root
// change, so the bound is never reached in practice; it exists so that no loop can spin forever.
constexpr int kUnionRetryLimit = 1 << 20;

// Returns false if the retry bound ran out (never expected; reported as an error flag).
__device__ __forceinline__ bool uf_unite(int32_t* parent, int32_t a, int32_t b, int limit = kUnionRetryLimit,
                                         int stride = 1)
{
  for (int it = 0; it < limit; ++it) {
    a = uf_find(parent, a, stride);
    b = uf_find(parent, b, stride);
    if (a == b) return true;
    if (a > b) {
      const int32_t t = a;
      a = b;
      b = t;
    }
    // hook the larger root under the smaller one
    const int32_t old = atomicCAS(parent + static_cast<int64_t>(b) * stride, b, a);
    if (old == b) return true;
    b = old;
  }
  return false;
}

// ---- launch descriptors shared by the orchestrator and the kernels ------------------------
// A slab of neighbour entries: entry q in [begin, end) links row[q] and col[q] (low 28 bits;
// the top 4 bits carry the entry's code in max-eps slabs).  begin/end are read on the device
// when begin_dev/end_dev are set (slabs compacted on the device), else begin = 0, end = count.
struct SlabRef {
  const int32_t* row = nullptr;
  const int32_t* col = nullptr;
  int64_t count = 0;
  const int64_t* begin_dev = nullptr;
  const int64_t* end_dev = nullptr;
};

// The slabs of one batch: annotated route, slab e = the entries of eps e (nslabs = k); direct
// route, slab 0 = the max-eps entries and an entry belongs to every eps >= its code.
struct MultiSlab {
  SlabRef s[kMaxEps];
  int nslabs = 0;
  int direct = 0;
};

struct DistLaunch {
  int64_t n;
  int32_t d, k;
  const float* xt;                 // dp x npad, dim-major
  const float* eps2;               // host, k values
  unsigned long long* counters;    // [0] pair cursor, [1] tile cursor
  uint64_t* edges;
  uint64_t edge_cap;
  int32_t* hist;                   // k x n
  int32_t* err;
  int sm_count;
  int shard = 0;                   // evaluate the shard-th of nshards equal tile-pair ranges
  int nshards = 1;
  const int32_t* perm = nullptr;   // XT column r holds point perm[r] (nullptr: identity)
  const long long* work = nullptr; // surviving tile pairs (nullptr: every tile pair)
  int64_t work_count = 0;
  const unsigned long long* work_count_dev = nullptr;  // count of `work` read on the device
                                                       // (the whole list, no sharding)
  const int64_t* work_total_dev = nullptr;  // screened pass: the worklist length on the device
  int64_t work_cap = 0;                     // (entries beyond work_cap were not written); each
                                            // shard's slice is computed on the device
  // Memory-bounded fit: only pairs with an endpoint at an XT position in [keep_lo, keep_hi) are
  // emitted (hist == nullptr then: the degrees are already known and are not counted again).
  int64_t keep_lo = 0;
  int64_t keep_hi = INT64_MAX;
};

// An emitted pair needs one endpoint (XT positions pi, pj) in [lo, hi).
__device__ __forceinline__ bool keep_pair(int64_t pi, int64_t pj, int64_t lo, int64_t hi)
{
  return (pi >= lo && pi < hi) || (pj >= lo && pj < hi);
}

// Screened distance pass (dist_tc.cu): tensor-core bound + exact chain for the candidates;
// tile pairs it cannot screen are appended to `fallback` (count in counters[5]) for
// launch_distance.  counters must hold 8 words: [0] edge cursor, [4] item cursor,
// [5] fallback count, [6] candidates, [7] screened tile pairs.
bool screen_supported(int32_t d, float eps2_max);
int32_t screen_rows(int32_t d);  // XT rows the screened pass reads (zero beyond d)
// Tensor map over the first `rows` rows of XT (dim-major, npad floats per row): boxes of
// {128 points, rows} (rows <= 256), zero-filled past n.
Status make_tile_map(const float* xt, int64_t n, int32_t rows, CUtensorMap* map);
Status launch_screened_distance(const DistLaunch& a, const float* box_lo, const float* box_hi, long long* fallback,
                                cudaStream_t s);

// ---- kernel launch accounting (host) --------------------------------------------------------
// Every kernel launch site calls count_launch(); dbm_stats.launches reports the difference
// over one fit (the bench's evidence that the native kernels ran).
int64_t count_launch(int64_t n = 1);
int64_t launches_so_far();

// ---- scans (host launchers, implemented in graph.cu) ------------------------------------
// exclusive scan of n int32 counts into n+1 int64 offsets (out[n] = total)
Status exclusive_scan_i32(const int32_t* in, int64_t* out, int64_t n, void* scratch,
                          size_t scratch_bytes, cudaStream_t s);
size_t scan_scratch_bytes(int64_t n);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace dbm
