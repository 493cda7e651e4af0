// api.cu -- fit_multi orchestrator and the C ABI of libdbm.so.
//
// Pass structure (B200 design; the reference's is runner_multi.cuh:549-749 / 771-1251):
//   1. Z-order, X -> XT (dim-major, padded) for TMA with the tile boxes, tile-pair prune.
//   2. One distance pass over the upper triangle of tile pairs: exact per-eps degree
//      histograms for every row and the list of neighbour pairs (i < j) within the largest
//      eps, each with its smallest-eps code.  If the pair buffer was too small the pass is
//      repeated once with the exact size (the counts are always complete).
//   3. Degrees, core counts (and the optional byte core masks), scan, symmetric max-eps CSR
//      with codes.
//   4. Batch plan: the reference's batch size for the budget, then its batch-correction
//      rule replayed on the measured per-batch nnz (runner_multi.cuh:1340-1456), and the
//      per-batch route (anotar_compensa or forced).
//   5. Labelling, batches ascending: the batched CC kernels for every owned config walk the
//      batch rows' max-eps entries and read each entry's eps from its code (dense batches on
//      the annotated route first compact the smaller eps' slabs, order-preserving, and walk
//      those instead: batch_compacts).
//   6. Roots -> ranks -> labels for all k*l configs at once.
#include "dbm_internal.cuh"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <limits>
#include <vector>

#ifndef DBM_GIT_SHA
#define DBM_GIT_SHA "unknown"
#endif
#ifndef DBM_BUILD_ID
#define DBM_BUILD_ID "unknown"
#endif

namespace dbm {

static std::atomic<int64_t> g_launches{0};
constexpr int64_t kOrderMinPoints = 4096;  // below this the spatial ordering does not pay
int64_t count_launch(int64_t n) { return g_launches.fetch_add(n) + n; }
int64_t launches_so_far() { return g_launches.load(); }

// launchers defined in dist.cu / graph.cu / cc.cu
Status launch_distance(const DistLaunch& a, cudaStream_t s);
Status transpose_pad(const float* x, float* xt, int64_t n, int32_t d, int32_t* err, cudaStream_t s,
                     const int32_t* perm = nullptr, int32_t rows = 0, float* box_lo = nullptr,
                     float* box_hi = nullptr);
int32_t padded_dims(int32_t d);
int64_t padded_points(int64_t n);
size_t order_scratch_bytes(int64_t n);
size_t prune_scratch_bytes(int64_t tiles, int32_t d);
size_t core_indices_scratch_bytes(int64_t n);
Status launch_core_indices(const uint8_t* core, int64_t n, int configs, int32_t* out, void* scratch,
                           size_t scratch_bytes, cudaStream_t s);
int64_t prune_units(int64_t tiles);
Status launch_tile_boxes(const float* xt, int64_t n, int64_t npad, int32_t d, float* lo, float* hi, cudaStream_t s);
Status launch_prune_count(int64_t tiles, const float* lo, const float* hi, int32_t d, float cutoff, void* scratch,
                          size_t scratch_bytes, void* scan_scratch, size_t scan_bytes, const int64_t** count_out_dev,
                          cudaStream_t s, const int32_t* ext_counts = nullptr);
Status launch_prune_write(int64_t tiles, const float* lo, const float* hi, int32_t d, float cutoff, void* scratch,
                          long long* work, int64_t cap, cudaStream_t s, const uint32_t* ext_masks = nullptr);
Status launch_prune_bound(int64_t tiles, const float* lo, const float* hi, int32_t d, float cutoff, int64_t u0,
                          int64_t u1, int32_t* counts, uint32_t* masks, cudaStream_t s);
int64_t prune_mask_words();
Status spatial_order(const float* x, int64_t n, int32_t d, int32_t* perm, void* scratch, size_t scratch_bytes,
                     cudaStream_t s, int64_t batch_rows = 0);
Status launch_degrees(const int32_t* hist, int64_t n, int k, const int32_t* minpts, int l,
                      int32_t* deg, int32_t* corecnt, int32_t* rowcnt, uint8_t* core_out,
                      uint8_t* corecnt8, cudaStream_t s);
Status launch_csr_scatter(const uint64_t* edges, int64_t m, int64_t n, const int64_t* off, int32_t* fill,
                          uint32_t* col, int32_t* row, cudaStream_t s);
Status launch_csr_scatter_batch(const uint64_t* edges, int64_t cap, const unsigned long long* m_dev, const int64_t* off,
                                int64_t s0, int64_t s1, int32_t* fill, uint32_t* col, int32_t* row, int32_t* err,
                                cudaStream_t s);
Status launch_batch_worklist(const long long* work, int64_t count, int64_t t0, int64_t t1, int32_t* flags,
                             int64_t* pos, void* scan_scratch, size_t scan_bytes, long long* out, cudaStream_t s);
Status launch_batch_nnz(const int64_t* off, int64_t n, int64_t bs, int64_t nb, int64_t* out,
                        cudaStream_t s);
Status launch_eps_totals(const int32_t* deg, int64_t n, int k, unsigned long long* out, int sm_count, cudaStream_t s);
Status launch_label_range(const int32_t* labels, int64_t total, int64_t n, unsigned long long* first_bad,
                          int sm_count, cudaStream_t s);
Status launch_cc_init(int64_t n, int k, int l, int32_t* G, int32_t* cur, unsigned long long* best,
                      cudaStream_t s);
Status launch_cc_batch(const MultiSlab& ms, int64_t upper_entries, int64_t n, int64_t rows, int k, int l,
                       int cfg_begin, int cfg_end, const int32_t* cc, const uint8_t* cc8, bool single_batch,
                       int32_t* G, int32_t* L,
                       unsigned long long* best, int32_t* cur, uint32_t tag, int32_t* err, int sm_count,
                       int union_limit, int32_t* snap, cudaStream_t s);
Status launch_slab_counts_all(const int32_t* deg, int64_t n, int ne, int64_t s0, int64_t rows, int32_t* counts,
                              cudaStream_t s);
Status launch_filter_all(const int64_t* off, const uint32_t* col, int64_t col_base, int64_t s0, int64_t rows, int ne,
                         const int64_t* off_flat, int32_t* col_flat, int32_t* row_flat, cudaStream_t s);
Status launch_cc_root_bits(int64_t n, int l, int c0, int c1, int64_t W, const int32_t* cc,
                           int32_t* G, uint32_t* words, int32_t* cnt, int sm_count, cudaStream_t s);
Status launch_cc_labels(int64_t n, int l, int c0, int c1, int64_t W, const int32_t* cc, int32_t* G,
                        const int32_t* cur, const uint32_t* words, const int64_t* wrank, int32_t* labels,
                        cudaStream_t s);

// ---- batch-size rules (runner_multi.cuh:79-119, 214-268, 437-499) --------------------------
struct Plan {
  uint64_t budget = 0;
  uint64_t batch_size = 0;
  int index_bits = 32;
  bool use_cuvs = true;
};

static uint64_t isz_of(int bits) { return bits == 64 ? 8 : 4; }

static uint64_t mem_per_row(int64_t n, int k, bool use_cuvs, int64_t hint, uint64_t isz)
{
  const uint64_t npr = hint > 0 ? static_cast<uint64_t>(hint) : static_cast<uint64_t>(n);
  if (use_cuvs) {
    const uint64_t per_entry = (k > 1 ? 2 : 1) * isz + (k > 1 ? 1 : 0);
    return static_cast<uint64_t>(n) + npr * per_entry + 2 * isz + static_cast<uint64_t>(k) * isz;
  }
  return 2ull * static_cast<uint64_t>(n) + (npr + 2) * isz + static_cast<uint64_t>(k) * isz;
}

static uint64_t mem_fixed(int64_t n, int k, int l, uint64_t isz)
{
  return static_cast<uint64_t>(n) * static_cast<uint64_t>(k) * static_cast<uint64_t>(l) +
         static_cast<uint64_t>(n) * isz * 2;
}

static Status batch_size_rule(int64_t n, int k, int l, uint64_t max_bytes, bool use_cuvs, int64_t hint,
                              int index_bits, uint64_t* out)
{
  const uint64_t isz = isz_of(index_bits);
  const uint64_t per_row = mem_per_row(n, k, use_cuvs, hint, isz);
  const uint64_t fixed = mem_fixed(n, k, l, isz);
  if (!(max_bytes > fixed))
    return Status::Err(DBM_ERR_FIXED_BUFFERS,
                       "insufficient memory for the fixed buffers: more than " +
                         std::to_string(fixed) + " bytes are needed for N=" + std::to_string(n) +
                         " and " + std::to_string(static_cast<long long>(k) * l) + " configurations");
  uint64_t bs = (max_bytes - fixed) / per_row;
  bs = std::min<uint64_t>(static_cast<uint64_t>(n), bs);
  if (bs < 1) bs = 1;
  const uint64_t imax = index_bits == 64 ? static_cast<uint64_t>(INT64_MAX)
                                         : static_cast<uint64_t>(INT32_MAX);
  const uint64_t cap = (imax - 1) / static_cast<uint64_t>(n);
  if (cap < 1)
    return Status::Err(DBM_ERR_INDEX_OVERFLOW,
                       "N=" + std::to_string(n) + " does not allow a single-row batch with the chosen index type");
  *out = std::min(bs, cap);
  return Status::Ok();
}

static uint64_t csr_bytes_per_entry(int k, bool use_cuvs, uint64_t isz)
{
  return (use_cuvs && k > 1) ? 2 * isz + 1 : isz;
}

static bool csr_fits(int64_t nnz, uint64_t per_entry, uint64_t available)
{
  return 1.1 * static_cast<double>(nnz) * static_cast<double>(per_entry) <= static_cast<double>(available);
}

static int64_t measured_degree(int64_t nnz, int64_t rows)
{
  const int64_t g = (nnz + rows - 1) / rows;
  return g > 1 ? g : 1;
}

static uint64_t csr_rows_that_fit(int64_t degree, uint64_t per_entry, uint64_t available)
{
  const uint64_t per_row = static_cast<uint64_t>(degree) * per_entry;
  const uint64_t fit = static_cast<uint64_t>(0.8 * static_cast<double>(available)) /
                       std::max<uint64_t>(1, per_row);
  return std::max<uint64_t>(1, fit);
}

static int annotate_pays(int64_t nnz, int64_t pairs, int k, int64_t d)
{
  const long double a = static_cast<long double>(nnz) * static_cast<long double>(d) * 40.0L;
  const long double b = static_cast<long double>(k - 1) *
                        (static_cast<long double>(pairs) * static_cast<long double>(d) + 60000000000.0L);
  return a < b;
}

// ---- workspace --------------------------------------------------------------------------------
struct Buffer {
  void* p = nullptr;
  size_t bytes = 0;
};

static Status ensure(Buffer& b, size_t bytes)
{
  if (bytes == 0) bytes = 256;
  if (b.bytes >= bytes) return Status::Ok();
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.bytes = 0;
  bytes = align_up(bytes, 256);
  cudaError_t e = cudaMalloc(&b.p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    b.p = nullptr;
    return Status::Err(DBM_ERR_OOM, "device allocation of " + std::to_string(bytes) +
                                      " bytes failed: " + cudaGetErrorString(e));
  }
  b.bytes = bytes;
  return Status::Ok();
}

template <typename T>
static T* as(Buffer& b) { return static_cast<T*>(b.p); }

}  // namespace dbm

struct dbm_handle {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int sm_count = 148;
  bool timing = false;
  struct PendingTimer {
    cudaEvent_t a, b;
    double* out;
  };
  std::vector<PendingTimer> pending_timers;  // phase events read after the call's final sync
  uint64_t edge_cap_hint = 0;
  int64_t work_cap_hint = 0;  // worklist capacity learned from earlier calls (no count sync then)
  // free device memory as of the last query (a cudaMemGetInfo costs ~1 ms of host time)
  size_t free_cached = 0, total_cached = 0;
  uint64_t free_cached_ws = 0;  // the handle's workspace bytes at that query
  std::chrono::steady_clock::time_point free_cached_at{};
  dbm::Buffer xt, hist, deg, cc, rowcnt, off, fill, edges, col, crow, minpts, counters, err;
  dbm::Buffer slab_counts, slab_off, slab_col, slab_row, G, L, best, cur, flags, rank, scan_scratch, bnnz;
  dbm::Buffer snap;  // root snapshot of dense batches (labelling)
  dbm::Buffer cc8;   // core counts as bytes (l <= 255)
  dbm::Buffer perm, order_scratch, box_lo, box_hi, prune_scratch, work, fallback;
  dbm::Buffer subwork, subflags, subpos;  // one batch's tile pairs (streamed fit)
  int distance_mode = DBM_DISTANCE_AUTO;
  int graph_mode = DBM_GRAPH_AUTO;
  int union_limit = dbm::kUnionRetryLimit;  // test knob (dbm_set_union_retry_limit)
  int64_t stream_work_count = 0;           // tile pairs of the batch-major worklist (streamed fit)
  dbm::Buffer xdev, labels_dev, core_dev;  // host-buffer entry point only
  int64_t* pinned = nullptr;               // small D2H staging
  size_t pinned_count = 0;

  uint64_t workspace_bytes() const
  {
    const dbm::Buffer* all[] = {&xt, &hist, &deg, &cc, &rowcnt, &off, &fill, &edges, &col, &crow,
                                &minpts, &counters, &err, &slab_counts, &slab_off, &slab_col,
                                &slab_row, &G, &L, &best, &cur, &flags, &rank, &scan_scratch, &bnnz,
                                &perm, &order_scratch, &box_lo, &box_hi, &prune_scratch,
                                &work, &fallback, &subwork, &subflags, &subpos, &snap, &cc8};
    uint64_t s = 0;
    for (auto* b : all) s += b->bytes;
    return s;
  }
};

namespace dbm {

static void set_err(char* err, size_t len, const std::string& msg)
{
  if (!err || len == 0) return;
  const size_t c = std::min(len - 1, msg.size());
  std::memcpy(err, msg.data(), c);
  err[c] = '\0';
}

static Status ensure_pinned(dbm_handle* h, size_t count)
{
  if (h->pinned_count >= count) return Status::Ok();
  if (h->pinned) cudaFreeHost(h->pinned);
  h->pinned = nullptr;
  h->pinned_count = 0;
  count = std::max<size_t>(count, 64);
  DBM_CUDA(cudaMallocHost(reinterpret_cast<void**>(&h->pinned), count * sizeof(int64_t)));
  h->pinned_count = count;
  return Status::Ok();
}

// Phase timing without extra synchronisation: events are recorded around a phase and read
// back after the call's final stream sync (resolve_phase_timers).
struct PhaseTimer {
  dbm_handle* h;
  cudaStream_t s;
  cudaEvent_t a = nullptr, b = nullptr;
  double* out;
  PhaseTimer(dbm_handle* h_, cudaStream_t s_, double* out_) : h(h_), s(s_), out(out_)
  {
    if (!h->timing || !out) return;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
      a = b = nullptr;
      return;
    }
    cudaEventRecord(a, s);
  }
  ~PhaseTimer()
  {
    if (!a) return;
    cudaEventRecord(b, s);
    h->pending_timers.push_back({a, b, out});
  }
};

static void resolve_phase_timers(dbm_handle* h)
{
  for (auto& t : h->pending_timers) {
    float ms = 0;
    if (cudaEventSynchronize(t.b) == cudaSuccess && cudaEventElapsedTime(&ms, t.a, t.b) == cudaSuccess)
      *t.out += ms;
    cudaEventDestroy(t.a);
    cudaEventDestroy(t.b);
  }
  h->pending_timers.clear();
}

static Status validate(int64_t n, int64_t d, const float* eps, int k, const int32_t* minpts, int l)
{
  if (n < 1) return Status::Err(DBM_ERR_INVALID, "No rows in the input array. DBSCAN cannot be fitted!");
  if (d < 1) return Status::Err(DBM_ERR_INVALID, "d must be >= 1");
  if (k < 1 || k > kMaxEps)
    return Status::Err(DBM_ERR_INVALID, "the number of eps values must be between 1 and 16");
  if (l < 1) return Status::Err(DBM_ERR_INVALID, "At least one minPts value is required");
  if (!eps || !minpts) return Status::Err(DBM_ERR_INVALID, "eps and minPts lists are required");
  const float safe = std::sqrt(std::numeric_limits<float>::max());
  for (int e = 0; e < k; ++e) {
    if (!std::isfinite(eps[e]) || eps[e] <= 0.0f || eps[e] > safe)
      return Status::Err(DBM_ERR_INVALID, "eps values must be finite, positive and not overflow eps^2");
    if (e > 0 && !(eps[e] > eps[e - 1]))
      return Status::Err(DBM_ERR_INVALID, "eps values must be strictly ascending (sort and deduplicate)");
  }
  for (int m = 0; m < l; ++m) {
    if (minpts[m] <= 0) return Status::Err(DBM_ERR_INVALID, "min-samples values must be positive");
    if (m > 0 && !(minpts[m] > minpts[m - 1]))
      return Status::Err(DBM_ERR_INVALID, "min-samples values must be strictly ascending (sort and deduplicate)");
  }
  if (n >= (int64_t(1) << kCodeShift))
    return Status::Err(DBM_ERR_TOO_LARGE, "N must be below 2^28");
  if (d > (int64_t(1) << 20)) return Status::Err(DBM_ERR_TOO_LARGE, "D must be below 2^20");
  return Status::Ok();
}

static Status read_err_flag(dbm_handle* h, cudaStream_t s)
{
  DBM_TRY(ensure_pinned(h, 4));
  h->pinned[0] = 0;
  DBM_CUDA(cudaMemcpyAsync(h->pinned, h->err.p, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  DBM_CUDA(cudaStreamSynchronize(s));
  const int32_t f = static_cast<int32_t>(h->pinned[0] & 0xffffffff);
  if (f & kErrTmaTimeout)
    return Status::Err(DBM_ERR_NOT_CONVERGED, "a bounded TMA wait in the distance kernel ran out");
  if (f & kErrUnionLimit)
    return Status::Err(DBM_ERR_NOT_CONVERGED, "union-find retry bound ran out");
  if (f & kErrGraphMismatch)
    return Status::Err(DBM_ERR_CUDA, "a row batch's neighbour pairs disagree with the degree pass");
  return Status::Ok();
}

// Degree-only pass: the distance kernel with no room for pairs still counts every pair.
static Status neighbor_counts(dbm_handle* h, const float* x, int64_t n, int64_t d, const float* eps,
                              int k, int32_t* deg_out, cudaStream_t s)
{
  const int32_t one = 1;
  DBM_TRY(validate(n, d, eps, k, &one, 1));
  if (!x || !deg_out) return Status::Err(DBM_ERR_INVALID, "x and deg must be device pointers");
  DBM_CUDA(cudaSetDevice(h->device));
  float eps2[kMaxEps];
  for (int e = 0; e < k; ++e) {
    volatile float v = eps[e] * eps[e];
    eps2[e] = v;
  }
  const int32_t di = static_cast<int32_t>(d);
  const int64_t kn = static_cast<int64_t>(k) * n;
  DBM_TRY(ensure(h->xt, sizeof(float) * static_cast<size_t>(padded_dims(di)) * padded_points(n)));
  DBM_TRY(ensure(h->hist, sizeof(int32_t) * kn));
  DBM_TRY(ensure(h->cc, sizeof(int32_t) * kn));
  DBM_TRY(ensure(h->rowcnt, sizeof(int32_t) * n));
  DBM_TRY(ensure(h->minpts, sizeof(int32_t)));
  DBM_TRY(ensure(h->counters, 4 * sizeof(unsigned long long)));
  DBM_TRY(ensure(h->err, 16));
  DBM_TRY(ensure(h->edges, sizeof(uint64_t)));
  DBM_CUDA(cudaMemcpyAsync(h->minpts.p, &one, sizeof(int32_t), cudaMemcpyHostToDevice, s));
  DBM_CUDA(cudaMemsetAsync(h->err.p, 0, 16, s));
  DBM_CUDA(cudaMemsetAsync(h->hist.p, 0, sizeof(int32_t) * kn, s));
  DBM_CUDA(cudaMemsetAsync(h->counters.p, 0, 4 * sizeof(unsigned long long), s));
  DBM_TRY(transpose_pad(x, as<float>(h->xt), n, di, as<int32_t>(h->err), s));
  DistLaunch a{n, di, k, as<float>(h->xt), eps2, as<unsigned long long>(h->counters),
               as<uint64_t>(h->edges), 0, as<int32_t>(h->hist), as<int32_t>(h->err), h->sm_count, 0, 1};
  DBM_TRY(launch_distance(a, s));
  DBM_TRY(launch_degrees(as<int32_t>(h->hist), n, k, as<int32_t>(h->minpts), 1, deg_out,
                         as<int32_t>(h->cc), as<int32_t>(h->rowcnt), nullptr, nullptr, s));
  DBM_TRY(ensure_pinned(h, 4));
  h->pinned[0] = 0;
  DBM_CUDA(cudaMemcpyAsync(h->pinned, h->err.p, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  DBM_CUDA(cudaStreamSynchronize(s));
  if (h->pinned[0] & kErrNonFinite) return Status::Err(DBM_ERR_NONFINITE, "the input contains NaN or infinity");
  if (h->pinned[0] & kErrTmaTimeout)
    return Status::Err(DBM_ERR_NOT_CONVERGED, "a bounded TMA wait in the distance kernel ran out");
  return Status::Ok();
}

static void square_eps(const float* eps, int k, float* eps2)
{
  for (int e = 0; e < k; ++e) {
    volatile float v = eps[e] * eps[e];  // float product, as the reference's host does
    eps2[e] = v;
  }
}

// Free device memory, as cudaMemGetInfo reports it.  The query is cached on the handle for up to
// one second and corrected by the handle's own workspace growth since then (the only
// allocations this library makes); another process allocating in that second is the one case a
// fresh query would see differently.
static Status free_memory(dbm_handle* h, size_t* free_b, size_t* total_b)
{
  const auto now = std::chrono::steady_clock::now();
  const uint64_t ws = h->workspace_bytes();
  if (h->total_cached == 0 || now - h->free_cached_at > std::chrono::seconds(1) || ws < h->free_cached_ws) {
    DBM_CUDA(cudaMemGetInfo(&h->free_cached, &h->total_cached));
    h->free_cached_at = now;
    h->free_cached_ws = ws;
  }
  const uint64_t grown = ws - h->free_cached_ws;
  *free_b = h->free_cached > grown ? h->free_cached - grown : 0;
  *total_b = h->total_cached;
  return Status::Ok();
}

// Budget, index width and the first batch-size check (runner_multi.cuh:1315-1337, 458-499).
static Status plan_budget(dbm_handle* h, int64_t n, int k, int l, const dbm_options& opt, dbm_stats& st,
                          Plan& plan)
{
  plan.use_cuvs = opt.backend != DBM_BACKEND_CODES;
  plan.index_bits = opt.index_bits == 64 ? 64
                    : opt.index_bits == 32 ? 32
                    : (static_cast<long double>(n) * n >= static_cast<long double>(INT32_MAX) ? 64 : 32);
  if (opt.max_bytes_per_batch == 0) {
    size_t free_b = 0, total_b = 0;
    DBM_TRY(free_memory(h, &free_b, &total_b));
    const uint64_t reusable = h->workspace_bytes();
    const uint64_t used = total_b - std::min<uint64_t>(total_b, free_b);
    const uint64_t available = reusable > used ? total_b : std::min<uint64_t>(total_b, free_b + reusable);
    plan.budget = 80 * available / 100;
  } else {
    plan.budget = opt.max_bytes_per_batch;
  }
  st.max_bytes_per_batch = plan.budget;
  st.index_bits = plan.index_bits;
  uint64_t bs0 = 0;
  return batch_size_rule(n, k, l, plan.budget, plan.use_cuvs, opt.neigh_per_row, plan.index_bits, &bs0);
}

// Distance pass over one shard of the tile pairs into hist (zeroed here) and h->edges.
// Keep masks and counts of every prune unit, gathered from the ranks of a multi-GPU fit that each
// bounded a share of the units (dbm_distance_prune_units); the order, XT and tile boxes are
// already in the handle then.
struct PruneInput {
  const int32_t* counts = nullptr;
  const uint32_t* masks = nullptr;
};

static bool screen_applies(const dbm_handle* h, int64_t n, int32_t d, const float* eps2, int k)
{
  return n >= kOrderMinPoints && h->distance_mode != DBM_DISTANCE_EXACT && screen_supported(d, eps2[k - 1]);
}

// Order, XT and tile boxes (the prune's inputs) for n >= kOrderMinPoints.
static Status distance_prepare(dbm_handle* h, const float* x, int64_t n, int32_t di, bool screen, cudaStream_t s)
{
  const int32_t xt_rows = screen ? std::max(padded_dims(di), screen_rows(di)) : padded_dims(di);
  const int64_t T = ceil_div(n, 128);
  DBM_TRY(ensure(h->perm, sizeof(int32_t) * n));
  DBM_TRY(ensure(h->order_scratch, order_scratch_bytes(n)));
  DBM_TRY(spatial_order(x, n, di, as<int32_t>(h->perm), h->order_scratch.p, h->order_scratch.bytes, s));
  DBM_TRY(ensure(h->box_lo, sizeof(float) * static_cast<size_t>(T) * di));
  DBM_TRY(ensure(h->box_hi, sizeof(float) * static_cast<size_t>(T) * di));
  // XT and the tile boxes (written by the transpose while each tile is in shared memory)
  return transpose_pad(x, as<float>(h->xt), n, di, as<int32_t>(h->err), s, as<int32_t>(h->perm), xt_rows,
                       as<float>(h->box_lo), as<float>(h->box_hi));
}

// With regrow, a pair buffer that turns out too small is grown to the exact count and the pass
// repeated; without, the call returns after one pass with *found_out > *cap_out (the histograms are
// complete either way, the pair list only when found <= cap).
static Status distance_stage(dbm_handle* h, const float* x, int64_t n, int64_t d, const float* eps2, int k,
                             int shard, int nshards, int32_t* hist, uint64_t cap_hint, uint64_t* found_out,
                             dbm_stats& st, cudaStream_t s, bool regrow = true, uint64_t* cap_out = nullptr,
                             const PruneInput* pre = nullptr)
{
  const int32_t di = static_cast<int32_t>(d);
  const int64_t kn = static_cast<int64_t>(k) * n;
  // Screened pass (dist_tc.cu) when the worklist exists (ordered points) and the bound applies;
  // the exact tile kernel takes the tile pairs it hands back, or everything when it is off.
  const bool screen = screen_applies(h, n, di, eps2, k);
  if (h->distance_mode == DBM_DISTANCE_SCREENED && !screen)
    return Status::Err(DBM_ERR_INVALID, "the screened distance pass needs N >= 4096, D <= 64 and eps^2 >= 1e-20");
  const int32_t xt_rows = screen ? std::max(padded_dims(di), screen_rows(di)) : padded_dims(di);
  DBM_TRY(ensure(h->xt, sizeof(float) * static_cast<size_t>(xt_rows) * padded_points(n)));
  DBM_TRY(ensure(h->counters, 8 * sizeof(unsigned long long)));
  DBM_TRY(ensure(h->err, 16));
  DBM_TRY(ensure_pinned(h, 16));
  if (!pre) DBM_CUDA(cudaMemsetAsync(h->err.p, 0, 16, s));
  PhaseTimer t(h, s, &st.ms_distance);
  // Z-order of the leading coordinates makes tiles spatially coherent, which lets whole warps
  // stop early in the distance kernel; results do not depend on the order.
  const int32_t* perm = nullptr;
  if (n >= kOrderMinPoints) {
    if (!pre) DBM_TRY(distance_prepare(h, x, n, di, screen, s));
    perm = as<int32_t>(h->perm);
  } else {
    DBM_TRY(transpose_pad(x, as<float>(h->xt), n, di, as<int32_t>(h->err), s, nullptr, xt_rows));
  }
  // Exact tile-pair pruning by per-tile bounding boxes (prune.cu): only tile pairs that may hold
  // a neighbour pair are evaluated.  Every rank builds the same worklist and takes its slice.
  const int64_t T = ceil_div(n, 128);
  const int64_t pairs = T * (T + 1) / 2;
  const long long* work = nullptr;
  int64_t work_count = 0, work_cap = 0;
  const int64_t* count_dev = nullptr;
  if (perm) {
    DBM_TRY(ensure(h->prune_scratch, prune_scratch_bytes(T, di)));
    DBM_TRY(ensure(h->scan_scratch, scan_scratch_bytes(prune_units(T) + 1)));
    DBM_TRY(launch_prune_count(T, as<float>(h->box_lo), as<float>(h->box_hi), di, eps2[k - 1], h->prune_scratch.p,
                               h->prune_scratch.bytes, h->scan_scratch.p, h->scan_scratch.bytes, &count_dev, s,
                               pre ? pre->counts : nullptr));
    if (screen && h->work_cap_hint > 0) {
      // the screen reads the worklist length on the device; a capacity learned from earlier
      // calls saves the host round trip (an overflow is seen at the pass's own sync below)
      work_cap = h->work_cap_hint;
    } else {
      h->pinned[0] = 0;
      DBM_CUDA(cudaMemcpyAsync(h->pinned, count_dev, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
      DBM_CUDA(cudaStreamSynchronize(s));
      work_count = h->pinned[0];
      work_cap = std::max<int64_t>(work_count, 1);
    }
    DBM_TRY(ensure(h->work, sizeof(long long) * work_cap));
    work_cap = static_cast<int64_t>(h->work.bytes / sizeof(long long));
    DBM_TRY(launch_prune_write(T, as<float>(h->box_lo), as<float>(h->box_hi), di, eps2[k - 1], h->prune_scratch.p,
                               as<long long>(h->work), work_cap, s, pre ? pre->masks : nullptr));
    work = as<long long>(h->work);
  }
  if (screen) DBM_TRY(ensure(h->fallback, sizeof(long long) * std::max<int64_t>(work_cap, 1)));
  uint64_t cap = std::max<uint64_t>(h->edge_cap_hint, cap_hint);
  uint64_t found = 0;
  for (int pass = 0; pass < 2; ++pass) {
    DBM_TRY(ensure(h->edges, sizeof(uint64_t) * std::max<uint64_t>(cap, 1)));
    cap = h->edges.bytes / sizeof(uint64_t);
    DBM_CUDA(cudaMemsetAsync(hist, 0, sizeof(int32_t) * kn, s));
    DBM_CUDA(cudaMemsetAsync(h->counters.p, 0, 8 * sizeof(unsigned long long), s));
    DistLaunch a{n, di, k, as<float>(h->xt), eps2, as<unsigned long long>(h->counters),
                 as<uint64_t>(h->edges), cap, hist, as<int32_t>(h->err), h->sm_count, shard, nshards, perm,
                 work, work_count};
    if (screen) {
      a.work_total_dev = count_dev;
      a.work_cap = work_cap;
      {
        PhaseTimer ts(h, s, &st.ms_screen);
        DBM_TRY(launch_screened_distance(a, as<float>(h->box_lo), as<float>(h->box_hi), as<long long>(h->fallback), s));
      }
      DistLaunch f = a;
      f.shard = 0;
      f.nshards = 1;
      f.work = as<long long>(h->fallback);
      f.work_count = 0;
      f.work_count_dev = as<unsigned long long>(h->counters) + 5;
      DBM_TRY(launch_distance(f, s));
    } else {
      DBM_TRY(launch_distance(a, s));
    }
    st.distance_passes = pass + 1;
    for (int w = 0; w < 10; ++w) h->pinned[w] = 0;
    DBM_CUDA(cudaMemcpyAsync(h->pinned, h->counters.p, 8 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s));
    DBM_CUDA(cudaMemcpyAsync(h->pinned + 8, h->err.p, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    if (count_dev) DBM_CUDA(cudaMemcpyAsync(h->pinned + 9, count_dev, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    DBM_CUDA(cudaStreamSynchronize(s));
    if (count_dev) {
      work_count = h->pinned[9];
      h->work_cap_hint = std::max<int64_t>(h->work_cap_hint, work_count + work_count / 8 + 1);
      if (work_count > work_cap) {
        // the worklist outgrew the learned capacity: redo the pass with the exact size (the
        // hint is now large enough, so this recursion ends after one level)
        return distance_stage(h, x, n, d, eps2, k, shard, nshards, hist, cap_hint, found_out, st, s, regrow, cap_out,
                              pre);
      }
    }
    st.tile_pairs_kept = !count_dev ? 1.0 : pairs > 0 ? static_cast<double>(work_count) / static_cast<double>(pairs) : 1.0;
    found = static_cast<uint64_t>(h->pinned[0]);
    {
      // exact-kernel work: 8 warps per 128 x 128 tile, each evaluating up to d dims for its
      // 16 x 128 pairs; the reference is this shard's share of all tile pairs
      const double full = static_cast<double>(pairs) / nshards * 8.0 * static_cast<double>(d);
      st.dist_work_fraction = full > 0 ? static_cast<double>(h->pinned[2]) / full : 1.0;
    }
    st.screened_tile_pairs = screen ? h->pinned[7] : 0;
    st.fallback_tile_pairs = screen ? h->pinned[5] : 0;
    st.screen_candidates = screen ? h->pinned[6] : 0;
    const int64_t flags = h->pinned[8] & 0xffffffff;
    if (flags & kErrNonFinite) return Status::Err(DBM_ERR_NONFINITE, "the input contains NaN or infinity");
    if (flags & kErrTmaTimeout)
      return Status::Err(DBM_ERR_NOT_CONVERGED, "a bounded wait in the distance kernels ran out");
    if (found <= cap || !regrow) break;
    if (pass == 1) return Status::Err(DBM_ERR_CUDA, "neighbour-pair buffer overflowed twice");
    cap = found;
  }
  if (found <= cap) h->edge_cap_hint = std::max<uint64_t>(h->edge_cap_hint, found);
  *found_out = found;
  if (cap_out) *cap_out = cap;
  return Status::Ok();
}

// ---- after the distance pass ------------------------------------------------------------------
// Batch plan of one fit: the reference's batch size for the budget, corrected on the measured
// per-batch nnz (runner_multi.cuh:1340-1456), and the per-batch routes.
struct BatchPlan {
  uint64_t bs = 0;
  int64_t nb = 0;
  std::vector<int64_t> bnnz;  // per batch, at the largest eps, self pairs included
  int64_t max_count = 0;      // largest per-batch entry count (self pairs excluded)
  int64_t rows(int64_t b, int64_t n) const
  {
    return std::min<int64_t>(n - b * static_cast<int64_t>(bs), static_cast<int64_t>(bs));
  }
};

// Degrees, core counts (and the optional byte core masks), CSR row offsets, batch plan and routes,
// from the complete per-code histograms.
static Status graph_prep(dbm_handle* h, int64_t n, int64_t d, int k, const int32_t* minpts, int l,
                         const int32_t* hist, uint8_t* core_out, const dbm_options& opt, const Plan& plan,
                         dbm_stats& st, std::vector<uint8_t>& routes, BatchPlan& bp, cudaStream_t s)
{
  const int64_t kn = static_cast<int64_t>(k) * n;
  const int64_t kln = kn * l;
  DBM_TRY(ensure(h->deg, sizeof(int32_t) * kn));
  DBM_TRY(ensure(h->cc, sizeof(int32_t) * kn));
  if (l <= 255) DBM_TRY(ensure(h->cc8, static_cast<size_t>(kn)));
  DBM_TRY(ensure(h->rowcnt, sizeof(int32_t) * n));
  DBM_TRY(ensure(h->off, sizeof(int64_t) * (n + 1)));
  DBM_TRY(ensure(h->fill, sizeof(int32_t) * n));
  DBM_TRY(ensure(h->minpts, sizeof(int32_t) * l));
  DBM_TRY(ensure(h->err, 16));
  DBM_TRY(ensure(h->scan_scratch, std::max(scan_scratch_bytes(n + 1), scan_scratch_bytes(kln + 1))));
  DBM_TRY(ensure_pinned(h, 16));
  DBM_CUDA(cudaMemcpyAsync(h->minpts.p, minpts, sizeof(int32_t) * l, cudaMemcpyHostToDevice, s));
  {
    PhaseTimer t(h, s, &st.ms_graph);
    DBM_TRY(launch_degrees(hist, n, k, as<int32_t>(h->minpts), l, as<int32_t>(h->deg), as<int32_t>(h->cc),
                           as<int32_t>(h->rowcnt), core_out, l <= 255 ? as<uint8_t>(h->cc8) : nullptr, s));
    DBM_TRY(exclusive_scan_i32(as<int32_t>(h->rowcnt), as<int64_t>(h->off), n, h->scan_scratch.p,
                               h->scan_scratch.bytes, s));
  }

  // ---- batch plan with the reference's correction rule ----
  const uint64_t isz = isz_of(plan.index_bits);
  const uint64_t per_entry = csr_bytes_per_entry(k, plan.use_cuvs, isz);
  uint64_t cap_rows = static_cast<uint64_t>(n);
  bool planned = false;
  for (int attempt = 0; attempt < 3 && !planned; ++attempt) {
    uint64_t rule_bs = 0;
    DBM_TRY(batch_size_rule(n, k, l, plan.budget, plan.use_cuvs, opt.neigh_per_row, plan.index_bits, &rule_bs));
    bp.bs = std::min(rule_bs, cap_rows);
    bp.nb = ceil_div(n, static_cast<int64_t>(bp.bs));
    st.attempts = attempt + 1;
    // per-batch nnz, then the per-eps entry totals, in one read-back
    DBM_TRY(ensure(h->bnnz, sizeof(int64_t) * (bp.nb + kMaxEps)));
    DBM_TRY(ensure_pinned(h, static_cast<size_t>(bp.nb + kMaxEps)));
    DBM_TRY(launch_batch_nnz(as<int64_t>(h->off), n, static_cast<int64_t>(bp.bs), bp.nb, as<int64_t>(h->bnnz), s));
    DBM_TRY(launch_eps_totals(as<int32_t>(h->deg), n, k, as<unsigned long long>(h->bnnz) + bp.nb, h->sm_count, s));
    DBM_CUDA(cudaMemcpyAsync(h->pinned, h->bnnz.p, sizeof(int64_t) * (bp.nb + k), cudaMemcpyDeviceToHost, s));
    DBM_CUDA(cudaStreamSynchronize(s));
    bp.bnnz.assign(h->pinned, h->pinned + bp.nb);
    for (int e = 0; e < k; ++e) st.nnz_per_eps[e] = h->pinned[bp.nb + e];
    uint64_t available = opt.csr_cap_bytes;
    if (available == 0) {
      size_t fr = 0, to = 0;
      DBM_TRY(free_memory(h, &fr, &to));
      available = fr;
    }
    int64_t measured = 0;
    if (plan.use_cuvs) {
      for (int64_t b = bp.nb - 1; b >= 0; --b) {
        if (!csr_fits(bp.bnnz[b], per_entry, available)) {
          measured = measured_degree(bp.bnnz[b], bp.rows(b, n));
          break;
        }
      }
    } else {
      const int64_t mx = *std::max_element(bp.bnnz.begin(), bp.bnnz.end());
      if (!csr_fits(mx, per_entry, available)) measured = measured_degree(mx, static_cast<int64_t>(bp.bs));
    }
    if (measured == 0) {
      planned = true;
      break;
    }
    st.batch_corrections += 1;
    const int64_t degree = attempt == 0 ? measured : n;
    const uint64_t new_cap = csr_rows_that_fit(degree, per_entry, available);
    if (!(new_cap < bp.bs))
      return Status::Err(DBM_ERR_CSR_NOT_FIT,
                         "the CSR does not fit in memory even with a batch of " + std::to_string(bp.bs) +
                           " rows (N=" + std::to_string(n) + ", measured degree " + std::to_string(measured) +
                           "); reduce --max-mbytes-per-batch or revisit eps");
    cap_rows = new_cap;
  }
  if (!planned) return Status::Err(DBM_ERR_CSR_NOT_FIT, "could not size the batch in 3 attempts");
  st.batch_size = bp.bs;
  st.batches = static_cast<int32_t>(bp.nb);
  routes.assign(static_cast<size_t>(bp.nb), DBM_BATCH_NOT_APPLICABLE);
  st.max_nnz = 0;
  st.total_nnz_max_eps = 0;
  bp.max_count = 0;
  for (int64_t b = 0; b < bp.nb; ++b) {
    const int64_t rows = bp.rows(b, n);
    st.max_nnz = std::max<int64_t>(st.max_nnz, bp.bnnz[b]);
    st.total_nnz_max_eps += bp.bnnz[b];
    bp.max_count = std::max<int64_t>(bp.max_count, bp.bnnz[b] - rows);
    if (plan.use_cuvs && k > 1) {
      const bool annotate = opt.route == DBM_ROUTE_ANNOTATED ? true
                            : opt.route == DBM_ROUTE_DENSE   ? false
                                                             : annotate_pays(bp.bnnz[b], n * rows, k, d);
      routes[b] = annotate ? DBM_BATCH_ANNOTATED : DBM_BATCH_DENSE;
      if (annotate) st.annotated_batches += 1; else st.dense_batches += 1;
    }
  }
  return Status::Ok();
}

// Whether batch b's labelling walks compacted per-eps slabs (the reference's annotated route,
// csr_multi_eps.cuh:194-234) or reads each max-eps entry's eps membership from its code.  The
// labels are the same either way.  Compaction (one pass over the max-eps entries) needs a call
// that owns a config of a smaller eps, and pays only for dense batches routed annotated: the
// walks then cover the smaller eps' entries once each instead of the max-eps entries once per
// eps.  Sparse batches walk directly: on C4 the per-batch compaction cost more than it saved,
// for the whole grid (labelling 2.10 -> 1.76 ms) and for a multi-GPU rank that owns only
// smaller-eps configs alike.  The reported route stays the reference's.
static bool batch_compacts(const BatchPlan& bp, const std::vector<uint8_t>& routes, int64_t b, int64_t n, int k,
                           int l, int cfg_begin)
{
  const int ne = k - 1;
  if (routes[b] == DBM_BATCH_DENSE || ne <= 0 || cfg_begin >= ne * l) return false;
  const int64_t rows = bp.rows(b, n);
  return bp.bnnz[b] - rows >= kDenseEntriesPerRow * rows;
}

// Bytes of the smaller-eps slabs the labelling compacts per batch (batch_compacts), sized by
// the largest batch.
static uint64_t slab_bytes(const BatchPlan& bp, const std::vector<uint8_t>& routes, int64_t n, int k, int l,
                           int cfg_begin)
{
  const int ne = k - 1;
  bool any = false;
  for (int64_t b = 0; b < bp.nb; ++b) any |= batch_compacts(bp, routes, b, n, k, l, cfg_begin);
  if (!any) return 0;
  return 2 * sizeof(int32_t) * static_cast<uint64_t>(std::max<int64_t>(bp.max_count, 1)) * ne +
         sizeof(int32_t) * bp.bs * ne + sizeof(int64_t) * (bp.bs * ne + 1);
}

// The whole symmetric max-eps CSR from the complete list of neighbour pairs.
static Status build_csr(dbm_handle* h, int64_t n, const uint64_t* edges, uint64_t found, dbm_stats& st, cudaStream_t s)
{
  PhaseTimer t(h, s, &st.ms_graph);
  DBM_TRY(ensure(h->col, sizeof(uint32_t) * 2 * std::max<uint64_t>(found, 1)));
  DBM_TRY(ensure(h->crow, sizeof(int32_t) * 2 * std::max<uint64_t>(found, 1)));
  DBM_CUDA(cudaMemsetAsync(h->fill.p, 0, sizeof(int32_t) * n, s));
  DBM_TRY(launch_csr_scatter(edges, static_cast<int64_t>(found), n, as<int64_t>(h->off), as<int32_t>(h->fill),
                             as<uint32_t>(h->col), as<int32_t>(h->crow), s));
  return Status::Ok();
}

// Where one batch's max-eps entries are: rows / cols of its `count` entries (col with the code
// in the top 4 bits), and the CSR position of col[0] (the per-eps compaction indexes col by CSR
// position).
struct BatchSlab {
  const int32_t* row = nullptr;
  const uint32_t* col = nullptr;
  int64_t col_base = 0;
};
using SlabSource = std::function<Status(int64_t b, int64_t s0, int64_t rows, int64_t base, BatchSlab& out)>;

// Labelling of the configs [cfg_begin, cfg_end), batches ascending; `source` yields each batch's
// max-eps entries.
static Status label_batches(dbm_handle* h, int64_t n, int k, int l, int cfg_begin, int cfg_end, const BatchPlan& bp,
                            const std::vector<uint8_t>& routes, dbm_stats& st, const SlabSource& source,
                            cudaStream_t s)
{
  const int64_t kln = static_cast<int64_t>(k) * l * n;
  const uint64_t bs = bp.bs;
  const int64_t nb = bp.nb;
  PhaseTimer t(h, s, &st.ms_label);
  DBM_TRY(ensure(h->G, sizeof(int32_t) * kln));
  DBM_TRY(ensure(h->cur, sizeof(int32_t) * kln));
  DBM_TRY(ensure(h->best, sizeof(unsigned long long) * kln));
  if (nb > 1) DBM_TRY(ensure(h->L, sizeof(int32_t) * kln));
  bool dense_any = false;
  for (int64_t b = 0; b < nb; ++b) dense_any |= bp.bnnz[b] - bp.rows(b, n) >= kDenseEntriesPerRow * bp.rows(b, n);
  if (dense_any) DBM_TRY(ensure(h->snap, kSnapBytesPerPoint * static_cast<uint64_t>(k) * n));
  const int ne = k - 1;  // smaller eps, compacted on the annotated route
  bool compacts = false;
  for (int64_t b = 0; b < nb; ++b) compacts |= batch_compacts(bp, routes, b, n, k, l, cfg_begin);
  if (compacts) {
    DBM_TRY(ensure(h->slab_counts, sizeof(int32_t) * bs * ne));
    DBM_TRY(ensure(h->slab_off, sizeof(int64_t) * (bs * ne + 1)));
    DBM_TRY(ensure(h->slab_col, sizeof(int32_t) * std::max<int64_t>(bp.max_count * ne, 1)));
    DBM_TRY(ensure(h->slab_row, sizeof(int32_t) * std::max<int64_t>(bp.max_count * ne, 1)));
    DBM_TRY(ensure(h->scan_scratch, scan_scratch_bytes(static_cast<int64_t>(bs) * ne + 1)));
  }
  DBM_TRY(launch_cc_init(n, k, l, as<int32_t>(h->G), as<int32_t>(h->cur),
                         as<unsigned long long>(h->best), s));
  int64_t base = 0;  // first max-eps CSR entry of the batch
  for (int64_t b = 0; b < nb; ++b) {
    const int64_t s0 = b * static_cast<int64_t>(bs);
    const int64_t rows = bp.rows(b, n);
    const int64_t count = bp.bnnz[b] - rows;  // entries without the self pairs
    const uint32_t tag = static_cast<uint32_t>(nb - 1 - b);
    BatchSlab slab;
    DBM_TRY(source(b, s0, rows, base, slab));
    SlabRef max_eps;
    max_eps.row = slab.row;
    max_eps.col = reinterpret_cast<const int32_t*>(slab.col);
    max_eps.count = count;
    MultiSlab ms;
    if (!batch_compacts(bp, routes, b, n, k, l, cfg_begin)) {
      // direct: eps membership straight from each max-eps entry's code, no per-eps copies
      ms.direct = 1;
      ms.nslabs = 1;
      ms.s[0] = max_eps;
    } else {
      // annotated: one pass compacts every smaller eps (order-preserving), then all slabs
      DBM_TRY(launch_slab_counts_all(as<int32_t>(h->deg), n, ne, s0, rows, as<int32_t>(h->slab_counts), s));
      DBM_TRY(exclusive_scan_i32(as<int32_t>(h->slab_counts), as<int64_t>(h->slab_off), rows * ne,
                                 h->scan_scratch.p, h->scan_scratch.bytes, s));
      DBM_TRY(launch_filter_all(as<int64_t>(h->off), slab.col, slab.col_base, s0, rows, ne, as<int64_t>(h->slab_off),
                                as<int32_t>(h->slab_col), as<int32_t>(h->slab_row), s));
      ms.direct = 0;
      ms.nslabs = k;
      for (int e = 0; e < ne; ++e) {
        ms.s[e].row = as<int32_t>(h->slab_row);
        ms.s[e].col = as<int32_t>(h->slab_col);
        ms.s[e].count = count;
        ms.s[e].begin_dev = as<int64_t>(h->slab_off) + static_cast<int64_t>(e) * rows;
        ms.s[e].end_dev = as<int64_t>(h->slab_off) + static_cast<int64_t>(e + 1) * rows;
      }
      ms.s[ne] = max_eps;
    }
    DBM_TRY(launch_cc_batch(ms, count, n, rows, k, l, cfg_begin, cfg_end, as<int32_t>(h->cc),
                            l <= 255 ? as<uint8_t>(h->cc8) : nullptr, nb == 1,
                            as<int32_t>(h->G), as<int32_t>(h->L), as<unsigned long long>(h->best),
                            as<int32_t>(h->cur), tag, as<int32_t>(h->err), h->sm_count, h->union_limit,
                            dense_any ? as<int32_t>(h->snap) : nullptr, s));
    base += count;
  }
  return Status::Ok();
}

// Roots -> ranks -> labels of the configs [cfg_begin, cfg_end), then the device error word.
static Status relabel_stage(dbm_handle* h, int64_t n, int k, int l, int cfg_begin, int cfg_end, int32_t* labels,
                            dbm_stats& st, cudaStream_t s)
{
  {
    PhaseTimer t(h, s, &st.ms_relabel);
    // roots as a bitmap (one 32-bit word per 32 points and config): the rank of a root is the
    // scan of the words' popcounts plus the bits below it, so the scan runs over n/32 words per
    // config instead of n flags
    const int64_t W = ceil_div(n, 32);
    const int64_t words_all = static_cast<int64_t>(k) * l * W, owned = static_cast<int64_t>(cfg_end - cfg_begin) * W;
    DBM_TRY(ensure(h->flags, sizeof(uint32_t) * static_cast<size_t>(words_all + owned)));
    DBM_TRY(ensure(h->rank, sizeof(int64_t) * static_cast<size_t>(owned + 1)));
    DBM_TRY(ensure(h->scan_scratch, scan_scratch_bytes(owned + 1)));
    uint32_t* words = as<uint32_t>(h->flags);
    int32_t* cnt = as<int32_t>(h->flags) + words_all;
    DBM_TRY(launch_cc_root_bits(n, l, cfg_begin, cfg_end, W, as<int32_t>(h->cc),
                                as<int32_t>(h->G), words, cnt, h->sm_count, s));
    DBM_TRY(exclusive_scan_i32(cnt, as<int64_t>(h->rank), owned, h->scan_scratch.p, h->scan_scratch.bytes, s));
    DBM_TRY(launch_cc_labels(n, l, cfg_begin, cfg_end, W, as<int32_t>(h->cc),
                             as<int32_t>(h->G), as<int32_t>(h->cur),
                             words, as<int64_t>(h->rank), labels, s));
  }
  return read_err_flag(h, s);
}

// Everything after the distance pass, from the complete per-code histograms and the complete
// list of neighbour pairs: degrees, core masks, CSR, batch plan, labelling of the configs
// [cfg_begin, cfg_end).
static Status label_stage(dbm_handle* h, int64_t n, int64_t d, int k, const int32_t* minpts, int l,
                          const int32_t* hist, const uint64_t* edges, uint64_t found, int cfg_begin,
                          int cfg_end, int32_t* labels, uint8_t* core_out, const dbm_options& opt,
                          const Plan& plan, dbm_stats& st, std::vector<uint8_t>& routes, cudaStream_t s)
{
  st.unique_pairs = n * (n - 1) / 2;
  st.edges = static_cast<int64_t>(found);
  BatchPlan bp;
  DBM_TRY(graph_prep(h, n, d, k, minpts, l, hist, core_out, opt, plan, st, routes, bp, s));
  DBM_TRY(build_csr(h, n, edges, found, st, s));
  const SlabSource whole = [&](int64_t, int64_t, int64_t, int64_t base, BatchSlab& out) {
    out.row = as<int32_t>(h->crow) + base;
    out.col = as<uint32_t>(h->col) + base;
    out.col_base = base;
    return Status::Ok();
  };
  DBM_TRY(label_batches(h, n, k, l, cfg_begin, cfg_end, bp, routes, st, whole, s));
  return relabel_stage(h, n, k, l, cfg_begin, cfg_end, labels, st, s);
}

// ---- memory-bounded fit: the graph one batch at a time ----------------------------------------
// Used when the whole max-eps pair list and CSR (24 bytes per neighbour pair, plus the per-batch
// slabs) would exceed the budget or the free memory.  The points are re-ordered batch-major (row
// batch, then Z-order), so the rows of batch b are the XT positions [s0, s1) and its tiles a
// contiguous range; per batch, the tile pairs touching that range are compacted from the pruned
// worklist, a distance pass emits only the pairs with an endpoint in the batch (the degrees are
// already complete, so no histogram is counted again), and the batch's rows of the CSR are built
// into buffers sized by the largest batch.  Each tile pair is evaluated by at most the two batches
// of its tiles.  The labelling kernels see exactly the entries the one-shot CSR holds for the
// batch, in another order, which no label depends on (min-index union-find).
static Status streamed_labels(dbm_handle* h, const float* x, int64_t n, int64_t d, const float* eps2, int k, int l,
                              int cfg_begin, int cfg_end, int32_t* labels, const BatchPlan& bp,
                              const std::vector<uint8_t>& routes, dbm_stats& st, cudaStream_t s)
{
  const int32_t di = static_cast<int32_t>(d);
  const bool screen = n >= kOrderMinPoints && h->distance_mode != DBM_DISTANCE_EXACT && screen_supported(di, eps2[k - 1]);
  const int32_t xt_rows = screen ? std::max(padded_dims(di), screen_rows(di)) : padded_dims(di);
  const int64_t T = ceil_div(n, 128);
  DBM_TRY(ensure(h->perm, sizeof(int32_t) * n));
  DBM_TRY(ensure(h->order_scratch, order_scratch_bytes(n)));
  DBM_TRY(ensure(h->xt, sizeof(float) * static_cast<size_t>(xt_rows) * padded_points(n)));
  DBM_TRY(ensure(h->box_lo, sizeof(float) * static_cast<size_t>(T) * di));
  DBM_TRY(ensure(h->box_hi, sizeof(float) * static_cast<size_t>(T) * di));
  DBM_TRY(ensure(h->prune_scratch, prune_scratch_bytes(T, di)));
  DBM_TRY(ensure(h->scan_scratch, scan_scratch_bytes(prune_units(T) + 1)));
  DBM_TRY(ensure(h->counters, 8 * sizeof(unsigned long long)));
  {
    PhaseTimer t(h, s, &st.ms_distance);
    DBM_TRY(spatial_order(x, n, di, as<int32_t>(h->perm), h->order_scratch.p, h->order_scratch.bytes, s,
                          static_cast<int64_t>(bp.bs)));
    DBM_TRY(transpose_pad(x, as<float>(h->xt), n, di, as<int32_t>(h->err), s, as<int32_t>(h->perm), xt_rows,
                          as<float>(h->box_lo), as<float>(h->box_hi)));
    const int64_t* count_dev = nullptr;
    DBM_TRY(launch_prune_count(T, as<float>(h->box_lo), as<float>(h->box_hi), di, eps2[k - 1], h->prune_scratch.p,
                               h->prune_scratch.bytes, h->scan_scratch.p, h->scan_scratch.bytes, &count_dev, s));
    h->pinned[0] = 0;
    DBM_CUDA(cudaMemcpyAsync(h->pinned, count_dev, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    DBM_CUDA(cudaStreamSynchronize(s));
    const int64_t W = std::max<int64_t>(h->pinned[0], 1);
    DBM_TRY(ensure(h->work, sizeof(long long) * W));
    DBM_TRY(launch_prune_write(T, as<float>(h->box_lo), as<float>(h->box_hi), di, eps2[k - 1], h->prune_scratch.p,
                               as<long long>(h->work), W, s));
    h->stream_work_count = h->pinned[0];
  }
  const int64_t W = h->stream_work_count;
  DBM_TRY(ensure(h->subwork, sizeof(long long) * std::max<int64_t>(W, 1)));
  DBM_TRY(ensure(h->subflags, sizeof(int32_t) * std::max<int64_t>(W, 1)));
  DBM_TRY(ensure(h->subpos, sizeof(int64_t) * (std::max<int64_t>(W, 1) + 1)));
  DBM_TRY(ensure(h->scan_scratch, scan_scratch_bytes(W + 1)));
  if (screen) DBM_TRY(ensure(h->fallback, sizeof(long long) * std::max<int64_t>(W, 1)));
  const uint64_t cap = static_cast<uint64_t>(std::max<int64_t>(bp.max_count, 1));
  DBM_TRY(ensure(h->edges, sizeof(uint64_t) * cap));
  DBM_TRY(ensure(h->col, sizeof(uint32_t) * cap));
  DBM_TRY(ensure(h->crow, sizeof(int32_t) * cap));
  st.streamed = 1;

  const SlabSource per_batch = [&](int64_t, int64_t s0, int64_t rows, int64_t base, BatchSlab& out) -> Status {
    const int64_t s1 = s0 + rows;
    auto* ctr = as<unsigned long long>(h->counters);
    DBM_CUDA(cudaMemsetAsync(ctr, 0, 8 * sizeof(unsigned long long), s));
    DBM_TRY(launch_batch_worklist(as<long long>(h->work), W, s0 / 128, ceil_div(s1, 128), as<int32_t>(h->subflags),
                                  as<int64_t>(h->subpos), h->scan_scratch.p, h->scan_scratch.bytes,
                                  as<long long>(h->subwork), s));
    const int64_t* sub_count = as<int64_t>(h->subpos) + W;
    DistLaunch a{n, di, k, as<float>(h->xt), eps2, ctr, as<uint64_t>(h->edges), cap, nullptr, as<int32_t>(h->err),
                 h->sm_count, 0, 1, as<int32_t>(h->perm), as<long long>(h->subwork), 0};
    a.keep_lo = s0;
    a.keep_hi = s1;
    if (screen) {
      a.work_total_dev = sub_count;
      a.work_cap = W;
      DBM_TRY(launch_screened_distance(a, as<float>(h->box_lo), as<float>(h->box_hi), as<long long>(h->fallback), s));
      DistLaunch f = a;
      f.work = as<long long>(h->fallback);
      f.work_count_dev = ctr + 5;
      DBM_TRY(launch_distance(f, s));
    } else {
      a.work_count_dev = reinterpret_cast<const unsigned long long*>(sub_count);
      DBM_TRY(launch_distance(a, s));
    }
    DBM_CUDA(cudaMemsetAsync(h->fill.p, 0, sizeof(int32_t) * rows, s));
    DBM_TRY(launch_csr_scatter_batch(as<uint64_t>(h->edges), static_cast<int64_t>(cap), ctr, as<int64_t>(h->off), s0,
                                     s1, as<int32_t>(h->fill), as<uint32_t>(h->col), as<int32_t>(h->crow),
                                     as<int32_t>(h->err), s));
    out.row = as<int32_t>(h->crow);
    out.col = as<uint32_t>(h->col);
    out.col_base = base;
    return Status::Ok();
  };
  DBM_TRY(label_batches(h, n, k, l, cfg_begin, cfg_end, bp, routes, st, per_batch, s));
  return relabel_stage(h, n, k, l, cfg_begin, cfg_end, labels, st, s);
}

static Status fit(dbm_handle* h, const float* x, int64_t n, int64_t d, const float* eps, int k,
                  const int32_t* minpts, int l, int32_t* labels, uint8_t* core_out,
                  const dbm_options& opt, dbm_stats& st, std::vector<uint8_t>& routes, cudaStream_t s)
{
  DBM_TRY(validate(n, d, eps, k, minpts, l));
  if (!x || !labels) return Status::Err(DBM_ERR_INVALID, "x and labels must be device pointers");
  DBM_CUDA(cudaSetDevice(h->device));
  Plan plan;
  DBM_TRY(plan_budget(h, n, k, l, opt, st, plan));
  float eps2[kMaxEps];
  square_eps(eps, k, eps2);
  DBM_TRY(ensure(h->hist, sizeof(int32_t) * static_cast<size_t>(k) * n));
  const uint64_t hint = static_cast<uint64_t>(n) *
                        static_cast<uint64_t>(opt.neigh_per_row > 0 ? opt.neigh_per_row : 16) / 2 + 1024;
  uint64_t found = 0, cap = 0;
  const bool forced = h->graph_mode == DBM_GRAPH_STREAMED;
  DBM_TRY(distance_stage(h, x, n, d, eps2, k, 0, 1, as<int32_t>(h->hist), forced ? 0 : hint, &found, st, s,
                         /*regrow=*/false, &cap));
  st.unique_pairs = n * (n - 1) / 2;
  st.edges = static_cast<int64_t>(found);
  BatchPlan bp;
  DBM_TRY(graph_prep(h, n, d, k, minpts, l, as<int32_t>(h->hist), core_out, opt, plan, st, routes, bp, s));
  bool stream = forced;
  if (!stream && h->graph_mode == DBM_GRAPH_AUTO) {
    // the whole pair list (when it outgrew its buffer), the whole CSR and the slabs are held
    // only if what they add to the workspace fits the budget and the free memory; otherwise the
    // graph is built one batch at a time
    size_t free_b = 0, total_b = 0;
    DBM_TRY(free_memory(h, &free_b, &total_b));
    const uint64_t ws = h->workspace_bytes();
    auto grow = [](uint64_t want, const Buffer& b) { return want > b.bytes ? want - b.bytes : uint64_t(0); };
    const uint64_t slabs = slab_bytes(bp, routes, n, k, l, 0);
    const uint64_t need = (found > cap ? grow(8 * found, h->edges) : 0) + grow(8 * found, h->col) +
                          grow(8 * found, h->crow) + grow(slabs, h->slab_col) / 2 + grow(slabs, h->slab_row) / 2;
    const uint64_t room = std::min<uint64_t>(plan.budget > ws ? plan.budget - ws : 0, free_b);
    stream = need > room;
  }
  if (stream) return streamed_labels(h, x, n, d, eps2, k, l, 0, k * l, labels, bp, routes, st, s);
  if (found > cap) {
    // one more pass with a pair buffer of the exact size (the histograms come out identical)
    const int32_t passes = st.distance_passes;
    DBM_TRY(distance_stage(h, x, n, d, eps2, k, 0, 1, as<int32_t>(h->hist), found, &found, st, s));
    st.distance_passes += passes;
  }
  DBM_TRY(build_csr(h, n, as<uint64_t>(h->edges), found, st, s));
  const SlabSource whole = [&](int64_t, int64_t, int64_t, int64_t base, BatchSlab& out) {
    out.row = as<int32_t>(h->crow) + base;
    out.col = as<uint32_t>(h->col) + base;
    out.col_base = base;
    return Status::Ok();
  };
  DBM_TRY(label_batches(h, n, k, l, 0, k * l, bp, routes, st, whole, s));
  return relabel_stage(h, n, k, l, 0, k * l, labels, st, s);
}

static dbm_options default_options()
{
  dbm_options o;
  std::memset(&o, 0, sizeof(o));
  o.backend = DBM_BACKEND_CUVS;
  return o;
}

}  // namespace dbm

// =============================================================================================
// C ABI
// =============================================================================================
extern "C" {

dbm_handle* dbm_create(int device, void* stream, char* err, size_t err_len)
{
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0 || device < 0 || device >= count) {
    cudaGetLastError();
    dbm::set_err(err, err_len, "no CUDA device " + std::to_string(device));
    return nullptr;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) {
    dbm::set_err(err, err_len, "device " + std::to_string(device) + " is not sm_100 class");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    dbm::set_err(err, err_len, "cudaSetDevice failed");
    return nullptr;
  }
  dbm_handle* h = new dbm_handle();
  h->device = device;
  h->sm_count = prop.multiProcessorCount;
  if (stream) {
    h->stream = static_cast<cudaStream_t>(stream);
  } else {
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete h;
      dbm::set_err(err, err_len, "cudaStreamCreate failed");
      return nullptr;
    }
    h->own_stream = true;
  }
  return h;
}

void dbm_destroy(dbm_handle* h)
{
  if (!h) return;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  dbm::Buffer* all[] = {&h->xt, &h->hist, &h->deg, &h->cc, &h->rowcnt, &h->off, &h->fill, &h->edges,
                        &h->col, &h->crow, &h->minpts, &h->counters, &h->err, &h->slab_counts,
                        &h->slab_off, &h->slab_col, &h->slab_row, &h->G, &h->L, &h->best, &h->cur,
                        &h->flags, &h->rank, &h->scan_scratch, &h->bnnz, &h->xdev, &h->labels_dev,
                        &h->core_dev, &h->perm, &h->order_scratch, &h->box_lo, &h->box_hi,
                        &h->prune_scratch, &h->work, &h->fallback, &h->subwork, &h->subflags, &h->subpos,
                        &h->snap, &h->cc8};
  for (auto* b : all)
    if (b->p) cudaFree(b->p);
  if (h->pinned) cudaFreeHost(h->pinned);
  if (h->own_stream) cudaStreamDestroy(h->stream);
  delete h;
}

uint64_t dbm_workspace_bytes(const dbm_handle* h) { return h ? h->workspace_bytes() : 0; }

void dbm_set_phase_timing(dbm_handle* h, int enabled)
{
  if (h) h->timing = enabled != 0;
}

int dbm_core_sample_indices(dbm_handle* h, const uint8_t* core_dev, int64_t n, int configs, int32_t* out_dev,
                            void* stream, char* err, size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  dbm::Status r;
  if (!core_dev || !out_dev || n < 1 || configs < 1 || n >= (int64_t(1) << 31))
    r = dbm::Status::Err(DBM_ERR_INVALID, "core mask and output are required, n in [1, 2^31), configs >= 1");
  if (r.ok()) {
    cudaSetDevice(h->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
    r = dbm::ensure(h->scan_scratch, dbm::core_indices_scratch_bytes(n));
    if (r.ok())
      r = dbm::launch_core_indices(core_dev, n, configs, out_dev, h->scan_scratch.p, h->scan_scratch.bytes, s);
    if (r.ok()) {
      const cudaError_t e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) r = dbm::Status::Err(DBM_ERR_CUDA, cudaGetErrorString(e));
    }
  }
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

int dbm_set_graph_mode(dbm_handle* h, int mode)
{
  if (!h || mode < DBM_GRAPH_AUTO || mode > DBM_GRAPH_STREAMED) return DBM_ERR_INVALID;
  h->graph_mode = mode;
  return DBM_OK;
}

int dbm_set_union_retry_limit(dbm_handle* h, int limit)
{
  if (!h || limit < 0) return DBM_ERR_INVALID;
  h->union_limit = limit == 0 ? 0 : std::min(limit, dbm::kUnionRetryLimit);
  return DBM_OK;
}

int dbm_set_distance_mode(dbm_handle* h, int mode)
{
  if (!h || mode < DBM_DISTANCE_AUTO || mode > DBM_DISTANCE_SCREENED) return DBM_ERR_INVALID;
  h->distance_mode = mode;
  return DBM_OK;
}

int dbm_fit_multi(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host,
                  int k, const int32_t* min_pts_host, int l, int32_t* labels_dev, uint8_t* core_dev,
                  const dbm_options* opt, dbm_stats* stats, uint8_t* batch_routes, int routes_len,
                  void* stream, char* err, size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  const dbm_options o = opt ? *opt : dbm::default_options();
  dbm_stats st;
  std::memset(&st, 0, sizeof(st));
  std::vector<uint8_t> routes;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  const int64_t launches0 = dbm::launches_so_far();
  dbm::Status r = dbm::fit(h, x_dev, n, d, eps_host, k, min_pts_host, l, labels_dev, core_dev, o, st,
                           routes, s);
  st.launches = static_cast<int32_t>(dbm::launches_so_far() - launches0);
  st.workspace_bytes = h->workspace_bytes();
  if (r.ok()) {
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) r = dbm::Status::Err(DBM_ERR_CUDA, cudaGetErrorString(e));
  }
  dbm::resolve_phase_timers(h);
  if (stats) *stats = st;
  if (batch_routes && routes_len > 0) {  // the batches only: the tail is left untouched
    const int nr = std::min(routes_len, static_cast<int>(routes.size()));
    for (int i = 0; i < nr; ++i) batch_routes[i] = routes[i];
  }
  if (!r.ok()) {
    dbm::set_err(err, err_len, r.msg);
    return r.code;
  }
  dbm::set_err(err, err_len, "");
  return DBM_OK;
}

int dbm_fit_multi_host(dbm_handle* h, const float* x_host, int64_t n, int64_t d,
                       const float* eps_host, int k, const int32_t* min_pts_host, int l,
                       int32_t* labels_host, uint8_t* core_host, const dbm_options* opt,
                       dbm_stats* stats, uint8_t* batch_routes, int routes_len, char* err,
                       size_t err_len)
{
  if (!h || !x_host || !labels_host || n < 1 || d < 1 || k < 1 || l < 1) {
    dbm::set_err(err, err_len, "invalid arguments");
    return DBM_ERR_INVALID;
  }
  cudaSetDevice(h->device);
  const size_t xb = sizeof(float) * static_cast<size_t>(n) * static_cast<size_t>(d);
  const size_t lb = sizeof(int32_t) * static_cast<size_t>(n) * k * l;
  dbm::Status r = dbm::ensure(h->xdev, xb);
  if (r.ok()) r = dbm::ensure(h->labels_dev, lb);
  if (r.ok() && core_host) r = dbm::ensure(h->core_dev, static_cast<size_t>(n) * k * l);
  if (!r.ok()) {
    dbm::set_err(err, err_len, r.msg);
    return r.code;
  }
  if (cudaMemcpyAsync(h->xdev.p, x_host, xb, cudaMemcpyHostToDevice, h->stream) != cudaSuccess) {
    dbm::set_err(err, err_len, "host-to-device copy of the points failed");
    return DBM_ERR_CUDA;
  }
  int rc = dbm_fit_multi(h, static_cast<const float*>(h->xdev.p), n, d, eps_host, k, min_pts_host, l,
                         static_cast<int32_t*>(h->labels_dev.p),
                         core_host ? static_cast<uint8_t*>(h->core_dev.p) : nullptr, opt, stats,
                         batch_routes, routes_len, h->stream, err, err_len);
  if (rc != DBM_OK) return rc;
  // range check on the device (-1 <= label < n), then the copies back
  const size_t total = static_cast<size_t>(n) * k * l;
  unsigned long long* first_bad = dbm::as<unsigned long long>(h->counters) + 3;
  if (cudaMemsetAsync(first_bad, 0xff, sizeof(unsigned long long), h->stream) != cudaSuccess ||
      !dbm::launch_label_range(static_cast<const int32_t*>(h->labels_dev.p), static_cast<int64_t>(total), n,
                               first_bad, h->sm_count, h->stream).ok()) {
    dbm::set_err(err, err_len, "label range check failed to launch");
    return DBM_ERR_CUDA;
  }
  unsigned long long bad = 0;
  if (cudaMemcpyAsync(&bad, first_bad, sizeof bad, cudaMemcpyDeviceToHost, h->stream) != cudaSuccess ||
      cudaMemcpyAsync(labels_host, h->labels_dev.p, lb, cudaMemcpyDeviceToHost, h->stream) != cudaSuccess ||
      (core_host && cudaMemcpyAsync(core_host, h->core_dev.p, static_cast<size_t>(n) * k * l,
                                    cudaMemcpyDeviceToHost, h->stream) != cudaSuccess) ||
      cudaStreamSynchronize(h->stream) != cudaSuccess) {
    dbm::set_err(err, err_len, "device-to-host copy of the labels failed");
    return DBM_ERR_CUDA;
  }
  if (bad != ~0ull) {
    dbm::set_err(err, err_len, "invalid CUDA label at position " + std::to_string(bad) + ": " +
                                 std::to_string(labels_host[bad]) + " (expected -1 <= label < " +
                                 std::to_string(n) + ")");
    return DBM_ERR_CUDA;
  }
  return DBM_OK;
}

int dbm_distance_shard(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host,
                       int k, int shard, int nshards, int32_t* hist_dev, uint64_t* edges_dev,
                       uint64_t edge_cap, uint64_t* edges_found, dbm_stats* stats, void* stream, char* err,
                       size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  const int32_t one = 1;
  dbm::Status r = dbm::validate(n, d, eps_host, k, &one, 1);
  if (r.ok() && (!x_dev || !hist_dev || !edges_found || nshards < 1 || shard < 0 || shard >= nshards))
    r = dbm::Status::Err(DBM_ERR_INVALID, "x, hist and edges_found are required and 0 <= shard < nshards");
  if (r.ok()) {
    cudaSetDevice(h->device);
    float eps2[dbm::kMaxEps];
    dbm::square_eps(eps_host, k, eps2);
    dbm_stats st;
    std::memset(&st, 0, sizeof(st));
    const int64_t launches0 = dbm::launches_so_far();
    uint64_t found = 0;
    r = dbm::distance_stage(h, x_dev, n, d, eps2, k, shard, nshards, hist_dev, edge_cap, &found, st, s);
    dbm::resolve_phase_timers(h);
    st.launches = static_cast<int32_t>(dbm::launches_so_far() - launches0);
    st.workspace_bytes = h->workspace_bytes();
    if (stats) *stats = st;
    if (r.ok()) {
      *edges_found = found;
      if (found <= edge_cap && found > 0) {
        const cudaError_t e = cudaMemcpyAsync(edges_dev, h->edges.p, found * sizeof(uint64_t),
                                              cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) cudaStreamSynchronize(s);
        else r = dbm::Status::Err(DBM_ERR_CUDA, cudaGetErrorString(e));
      }
    }
  }
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

int64_t dbm_prune_units(int64_t n)
{
  return n >= dbm::kOrderMinPoints ? dbm::prune_units(dbm::ceil_div(n, 128)) : 0;
}

int dbm_prune_mask_words(void) { return static_cast<int>(dbm::prune_mask_words()); }

int dbm_distance_prune_units(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host, int k,
                             int64_t unit_begin, int64_t unit_end, int32_t* counts_dev, uint32_t* masks_dev,
                             void* stream, char* err, size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  const int32_t one = 1;
  dbm::Status r = dbm::validate(n, d, eps_host, k, &one, 1);
  const int64_t units = dbm_prune_units(n);
  if (r.ok() && (!x_dev || !counts_dev || !masks_dev || units == 0 || unit_begin < 0 || unit_begin > unit_end ||
                 unit_end > units))
    r = dbm::Status::Err(DBM_ERR_INVALID, "x, counts and masks are required, N >= 4096 and 0 <= begin <= end <= units");
  if (r.ok()) {
    cudaSetDevice(h->device);
    float eps2[dbm::kMaxEps];
    dbm::square_eps(eps_host, k, eps2);
    const int32_t di = static_cast<int32_t>(d);
    const bool screen = dbm::screen_applies(h, n, di, eps2, k);
    const int32_t xt_rows = screen ? std::max(dbm::padded_dims(di), dbm::screen_rows(di)) : dbm::padded_dims(di);
    r = dbm::ensure(h->xt, sizeof(float) * static_cast<size_t>(xt_rows) * dbm::padded_points(n));
    if (r.ok()) r = dbm::ensure(h->err, 16);
    if (r.ok() && cudaMemsetAsync(h->err.p, 0, 16, s) != cudaSuccess)
      r = dbm::Status::Err(DBM_ERR_CUDA, "cudaMemsetAsync failed");
    if (r.ok()) r = dbm::distance_prepare(h, x_dev, n, di, screen, s);
    if (r.ok())
      r = dbm::launch_prune_bound(dbm::ceil_div(n, 128), dbm::as<float>(h->box_lo), dbm::as<float>(h->box_hi), di,
                                  eps2[k - 1], unit_begin, unit_end, counts_dev, masks_dev, s);
  }
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

int dbm_distance_shard_pruned(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host, int k,
                              int shard, int nshards, const int32_t* counts_dev, const uint32_t* masks_dev,
                              int32_t* hist_dev, uint64_t* edges_dev, uint64_t edge_cap, uint64_t* edges_found,
                              dbm_stats* stats, void* stream, char* err, size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  const int32_t one = 1;
  dbm::Status r = dbm::validate(n, d, eps_host, k, &one, 1);
  if (r.ok() && (!x_dev || !hist_dev || !edges_found || !counts_dev || !masks_dev || nshards < 1 || shard < 0 ||
                 shard >= nshards || dbm_prune_units(n) == 0))
    r = dbm::Status::Err(DBM_ERR_INVALID, "x, hist, counts, masks and edges_found are required, N >= 4096 and "
                                          "0 <= shard < nshards");
  if (r.ok()) {
    cudaSetDevice(h->device);
    float eps2[dbm::kMaxEps];
    dbm::square_eps(eps_host, k, eps2);
    dbm_stats st;
    std::memset(&st, 0, sizeof(st));
    const int64_t launches0 = dbm::launches_so_far();
    uint64_t found = 0;
    const dbm::PruneInput pre{counts_dev, masks_dev};
    r = dbm::distance_stage(h, x_dev, n, d, eps2, k, shard, nshards, hist_dev, edge_cap, &found, st, s, true, nullptr,
                            &pre);
    dbm::resolve_phase_timers(h);
    st.launches = static_cast<int32_t>(dbm::launches_so_far() - launches0);
    st.workspace_bytes = h->workspace_bytes();
    if (stats) *stats = st;
    if (r.ok()) {
      *edges_found = found;
      if (found <= edge_cap && found > 0) {
        const cudaError_t e = cudaMemcpyAsync(edges_dev, h->edges.p, found * sizeof(uint64_t),
                                              cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) cudaStreamSynchronize(s);
        else r = dbm::Status::Err(DBM_ERR_CUDA, cudaGetErrorString(e));
      }
    }
  }
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

int dbm_fit_multi_from_graph(dbm_handle* h, int64_t n, int64_t d, const float* eps_host, int k,
                             const int32_t* min_pts_host, int l, const int32_t* hist_dev,
                             const uint64_t* edges_dev, uint64_t m_edges, int cfg_begin, int cfg_end,
                             int32_t* labels_dev, uint8_t* core_dev, const dbm_options* opt,
                             dbm_stats* stats, uint8_t* batch_routes, int routes_len, void* stream,
                             char* err, size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  const dbm_options o = opt ? *opt : dbm::default_options();
  dbm_stats st;
  std::memset(&st, 0, sizeof(st));
  std::vector<uint8_t> routes;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  const int64_t launches0 = dbm::launches_so_far();
  dbm::Status r = dbm::validate(n, d, eps_host, k, min_pts_host, l);
  if (r.ok() && (!hist_dev || (!edges_dev && m_edges > 0) || !labels_dev || cfg_begin < 0 ||
                 cfg_end > k * l || cfg_begin > cfg_end))
    r = dbm::Status::Err(DBM_ERR_INVALID, "hist, edges and labels are required and 0 <= cfg_begin <= cfg_end <= k*l");
  if (r.ok()) {
    cudaSetDevice(h->device);
    dbm::Plan plan;
    r = dbm::plan_budget(h, n, k, l, o, st, plan);
    if (r.ok())
      r = dbm::label_stage(h, n, d, k, min_pts_host, l, hist_dev, edges_dev, m_edges, cfg_begin, cfg_end,
                           labels_dev, core_dev, o, plan, st, routes, s);
    if (r.ok()) {
      const cudaError_t e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) r = dbm::Status::Err(DBM_ERR_CUDA, cudaGetErrorString(e));
    }
  }
  dbm::resolve_phase_timers(h);
  st.launches = static_cast<int32_t>(dbm::launches_so_far() - launches0);
  st.workspace_bytes = h->workspace_bytes();
  if (stats) *stats = st;
  if (batch_routes && routes_len > 0) {  // the batches only: the tail is left untouched
    const int nr = std::min(routes_len, static_cast<int>(routes.size()));
    for (int i = 0; i < nr; ++i) batch_routes[i] = routes[i];
  }
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

int dbm_neighbor_counts(dbm_handle* h, const float* x_dev, int64_t n, int64_t d,
                        const float* eps_host, int k, int32_t* deg_dev, void* stream, char* err,
                        size_t err_len)
{
  if (!h) {
    dbm::set_err(err, err_len, "null handle");
    return DBM_ERR_INVALID;
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  dbm::Status r = dbm::neighbor_counts(h, x_dev, n, d, eps_host, k, deg_dev, s);
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

int dbm_batch_size(int64_t n, int k, int l, uint64_t max_bytes, int backend, int64_t neigh_per_row,
                   int index_bits, uint64_t* batch_size_out, char* err, size_t err_len)
{
  if (n < 1 || k < 1 || l < 1 || !batch_size_out) {
    dbm::set_err(err, err_len, "invalid arguments");
    return DBM_ERR_INVALID;
  }
  const int bits = index_bits == 64 ? 64 : index_bits == 32 ? 32 : dbm_auto_index_bits(n);
  dbm::Status r = dbm::batch_size_rule(n, k, l, max_bytes, backend != DBM_BACKEND_CODES,
                                       neigh_per_row, bits, batch_size_out);
  dbm::set_err(err, err_len, r.msg);
  return r.code;
}

uint64_t dbm_max_bytes_for_batch_size(int64_t n, int k, int l, uint64_t batch_size, int backend,
                                      int64_t neigh_per_row, int index_bits)
{
  const int bits = index_bits == 64 ? 64 : index_bits == 32 ? 32 : dbm_auto_index_bits(n);
  const uint64_t isz = dbm::isz_of(bits);
  return dbm::mem_fixed(n, k, l, isz) +
         batch_size * dbm::mem_per_row(n, k, backend != DBM_BACKEND_CODES, neigh_per_row, isz) + 1;
}

int dbm_annotate_pays(int64_t nnz, int64_t pairs, int k, int64_t d)
{
  return dbm::annotate_pays(nnz, pairs, k, d);
}

int dbm_auto_index_bits(int64_t n)
{
  return static_cast<long double>(n) * n >= static_cast<long double>(INT32_MAX) ? 64 : 32;
}

const char* dbm_build_info_json(void)
{
  return "{\"git_sha\":\"" DBM_GIT_SHA "\",\"revision_kind\":\"provided\",\"git_dirty\":null,"
         "\"build_id\":\"" DBM_BUILD_ID "\",\"cuda_arch\":\"sm_100a\","
         "\"configured_backend\":\"cuvs\",\"compiled_backends\":[\"cuvs\",\"codes\"],"
         "\"flags\":\"arch=sm_100a,O3,fmad=default\","
         "\"neighborhood_kernel\":\"dbm-sm100a-fp32-triangle-tma\"}";
}

}  // extern "C"
