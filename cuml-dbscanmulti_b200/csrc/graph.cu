// graph.cu -- degrees, core counts, scans and CSR construction (HBM-bound integer kernels).
//
// Reference counterparts (Math-BUG/cuML-DBSCANMulti):
//   degrees_kernel       per-eps degree vectors vd[e] (eps_neighborhood.cuh:171-174, 370-378)
//                        and the k*l core masks (corepoints_multi.cuh:86-123): a point is core
//                        for (e, m) iff degree_e >= minPts[m]; with minPts ascending that is
//                        m < corecnt[e][i].
//   exclusive_scan_i32   thrust::exclusive_scan of the degrees (csr_multi_eps.cuh:320-323,
//                        third_party/cuml/cpp/src/dbscan/adjgraph/algo.cuh:54)
//   csr_scatter_kernel   the max-eps CSR with a code per entry that the reference builds with
//                        adj_to_csr + annotateKernel (adjgraph/algo.cuh:56-57,
//                        csr_multi_eps.cuh:93-185); here it is filled straight from the
//                        neighbour pairs the distance kernel emitted, both directions.
//   filter_all_kernel    order-preserving per-row compaction of the max-eps CSR to every
//                        smaller eps in one pass (filterKernel, csr_multi_eps.cuh:194-234,
//                        runs once per eps): dense batches of the annotated route.
//   batch_nnz_kernel     per-batch nnz at the largest eps (runner_multi.cuh:898-904).
#include "dbm_internal.cuh"

#include <cub/device/device_select.cuh>
#include <thrust/iterator/counting_iterator.h>

#include <algorithm>

namespace dbm {

// ---- scan ---------------------------------------------------------------------------------
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int64_t kScanBlock = kScanThreads * kScanItems;

template <typename T>
__device__ __forceinline__ T block_exclusive_sum(T v, T* warp_sums, T& total)
{
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const T u = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += u;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    T w = (lane < (blockDim.x >> 5)) ? warp_sums[lane] : T(0);
    T wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const T u = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += u;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) warp_sums[32] = wi;
  }
  __syncthreads();
  const T res = warp_sums[warp] + incl - v;
  total = warp_sums[32];
  __syncthreads();
  return res;
}

__global__ void scan_partials_kernel(const int32_t* __restrict__ in, int64_t n,
                                     int64_t* __restrict__ partials)
{
  __shared__ int64_t ws[33];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanBlock + threadIdx.x * kScanItems;
  int64_t s = 0;
#pragma unroll
  for (int q = 0; q < kScanItems; ++q)
    if (base + q < n) s += in[base + q];
  int64_t total;
  block_exclusive_sum<int64_t>(s, ws, total);
  if (threadIdx.x == 0) partials[blockIdx.x] = total;
}

__global__ void scan_top_kernel(int64_t* __restrict__ partials, int64_t nparts)
{
  __shared__ int64_t ws[33];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t b0 = 0; b0 < nparts; b0 += kScanThreads) {
    const int64_t i = b0 + threadIdx.x;
    const int64_t v = i < nparts ? partials[i] : 0;
    int64_t total;
    const int64_t ex = block_exclusive_sum<int64_t>(v, ws, total);
    if (i < nparts) partials[i] = carry + ex;
    __syncthreads();
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) partials[nparts] = carry;
}

__global__ void scan_final_kernel(const int32_t* __restrict__ in, int64_t n,
                                  const int64_t* __restrict__ partials, int64_t* __restrict__ out,
                                  int64_t nparts)
{
  __shared__ int64_t ws[33];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanBlock + threadIdx.x * kScanItems;
  int64_t v[kScanItems];
  int64_t s = 0;
#pragma unroll
  for (int q = 0; q < kScanItems; ++q) {
    v[q] = (base + q < n) ? in[base + q] : 0;
    s += v[q];
  }
  int64_t total;
  int64_t ex = block_exclusive_sum<int64_t>(s, ws, total) + partials[blockIdx.x];
#pragma unroll
  for (int q = 0; q < kScanItems; ++q) {
    if (base + q < n) out[base + q] = ex;
    ex += v[q];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) out[n] = partials[nparts];
}

size_t scan_scratch_bytes(int64_t n) { return sizeof(int64_t) * (ceil_div(n, kScanBlock) + 2); }

Status exclusive_scan_i32(const int32_t* in, int64_t* out, int64_t n, void* scratch,
                          size_t scratch_bytes, cudaStream_t s)
{
  if (n <= 0) {
    DBM_CUDA(cudaMemsetAsync(out, 0, sizeof(int64_t), s));
    return Status::Ok();
  }
  const int64_t nparts = ceil_div(n, kScanBlock);
  if (scratch_bytes < scan_scratch_bytes(n))
    return Status::Err(DBM_ERR_INVALID, "scan scratch too small");
  int64_t* partials = static_cast<int64_t*>(scratch);
  count_launch();
  scan_partials_kernel<<<static_cast<unsigned>(nparts), kScanThreads, 0, s>>>(in, n, partials);
  count_launch();
  scan_top_kernel<<<1, kScanThreads, 0, s>>>(partials, nparts);
  count_launch();
  scan_final_kernel<<<static_cast<unsigned>(nparts), kScanThreads, 0, s>>>(in, n, partials, out,
                                                                          nparts);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// ---- degrees and core counts ----------------------------------------------------------------
// deg[e][i] = 1 + sum_{c <= e} hist[c][i]; corecnt[e][i] = #{m : deg >= minpts[m]};
// rowcnt[i] = deg[k-1][i] - 1 (max-eps neighbours without the point itself); corecnt8 (optional,
// l <= 255): the core counts as bytes, a quarter of the cache footprint for the labelling's
// gathers.
__global__ void degrees_kernel(const int32_t* __restrict__ hist, int64_t n, int k,
                               const int32_t* __restrict__ minpts, int l, int32_t* __restrict__ deg,
                               int32_t* __restrict__ corecnt, int32_t* __restrict__ rowcnt,
                               uint8_t* __restrict__ core_out, uint8_t* __restrict__ corecnt8)
{
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int32_t run = 1;
  for (int e = 0; e < k; ++e) {
    run += hist[static_cast<int64_t>(e) * n + i];
    deg[static_cast<int64_t>(e) * n + i] = run;
    // minpts ascending: count of thresholds <= run by binary search
    int lo = 0, hi = l;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(minpts + mid) <= run) lo = mid + 1; else hi = mid;
    }
    corecnt[static_cast<int64_t>(e) * n + i] = lo;
    if (corecnt8) corecnt8[static_cast<int64_t>(e) * n + i] = static_cast<uint8_t>(lo);
    if (core_out) {
      for (int m = 0; m < l; ++m)
        core_out[(static_cast<int64_t>(e) * l + m) * n + i] = static_cast<uint8_t>(m < lo);
    }
  }
  rowcnt[i] = run - 1;
}

Status launch_degrees(const int32_t* hist, int64_t n, int k, const int32_t* minpts, int l,
                      int32_t* deg, int32_t* corecnt, int32_t* rowcnt, uint8_t* core_out,
                      uint8_t* corecnt8, cudaStream_t s)
{
  count_launch();
  degrees_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(
    hist, n, k, minpts, l, deg, corecnt, rowcnt, core_out, l <= 255 ? corecnt8 : nullptr);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// ---- max-eps CSR from the neighbour pairs ---------------------------------------------------
// Slot claims on the per-row cursors: the lanes of a warp that hold the same row share one
// atomic (the distance pass emits each thread's pairs row by row, so a warp of consecutive pairs
// holds a few rows many times in a dense graph) and take consecutive slots.  A lane holding
// kNoRow claims nothing.  All 32 lanes must call it.
constexpr uint32_t kNoRow = 0xffffffffu;

__device__ __forceinline__ int32_t warp_claim(int32_t* fill, uint32_t v)
{
  const unsigned peers = __match_any_sync(0xffffffffu, v);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(peers) - 1;
  int32_t base = 0;
  if (lane == leader && v != kNoRow) base = atomicAdd(fill + v, __popc(peers));
  base = __shfl_sync(0xffffffffu, base, leader);
  return base + __popc(peers & ((1u << lane) - 1u));
}

// row[q - off[s0]] = r for every CSR position q of the rows r in [s0, s1) (at most cap positions):
// `lanes` consecutive lanes (a power of two <= 32, about the mean row length) per row, so the
// stores of a warp are contiguous whether rows hold 4 entries or 40,000.  The scatter kernels
// write only the columns: a row's entries are contiguous, so its row ids need no scattered
// 4-byte stores.
__global__ void csr_rows_kernel(const int64_t* __restrict__ off, int64_t s0, int64_t s1, int64_t cap, int lanes,
                                int32_t* __restrict__ row)
{
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t groups = (static_cast<int64_t>(gridDim.x) * blockDim.x) / lanes;
  const int sub = static_cast<int>(t % lanes);
  const int64_t base = off[s0];
  for (int64_t r = s0 + t / lanes; r < s1; r += groups) {
    const int64_t beg = off[r] - base;
    const int64_t end = off[r + 1] - base < cap ? off[r + 1] - base : cap;
    for (int64_t q = beg + sub; q < end; q += lanes) row[q] = static_cast<int32_t>(r);
  }
}

// entries: the expected number of CSR positions of the rows (sets the lanes per row)
static Status launch_csr_rows(const int64_t* off, int64_t s0, int64_t s1, int64_t cap, int64_t entries, int32_t* row,
                              cudaStream_t s)
{
  if (s1 <= s0 || cap <= 0) return Status::Ok();
  const int64_t mean = ceil_div(std::max<int64_t>(entries, 1), s1 - s0);
  int lanes = 1;
  while (lanes < 32 && lanes < mean) lanes <<= 1;
  const int64_t blocks = std::min<int64_t>(ceil_div((s1 - s0) * lanes, 256), int64_t(1) << 20);
  count_launch();
  csr_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(off, s0, s1, cap, lanes, row);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// grid: whole warps (blocks of 256); lanes past m take part in the claims only
__global__ void csr_scatter_kernel(const uint64_t* __restrict__ edges, int64_t m,
                                   const int64_t* __restrict__ off, int32_t* __restrict__ fill,
                                   uint32_t* __restrict__ col)
{
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool valid = q < m;
  const uint64_t w = valid ? edges[q] : 0;
  const uint32_t i = static_cast<uint32_t>(w >> 32);
  const uint32_t lo = static_cast<uint32_t>(w);
  const uint32_t j = lo & kColMask;
  const uint32_t code = lo & ~kColMask;
  const int32_t ki = warp_claim(fill, valid ? i : kNoRow);
  const int32_t kj = warp_claim(fill, valid ? j : kNoRow);
  if (!valid) return;
  col[off[i] + ki] = code | j;
  col[off[j] + kj] = code | i;
}

// the max-eps CSR of all n rows (2 m entries): columns scattered from the pairs, row ids per row
Status launch_csr_scatter(const uint64_t* edges, int64_t m, int64_t n, const int64_t* off, int32_t* fill,
                          uint32_t* col, int32_t* row, cudaStream_t s)
{
  if (m <= 0) return Status::Ok();
  count_launch();
  csr_scatter_kernel<<<static_cast<unsigned>(ceil_div(m, 256)), 256, 0, s>>>(edges, m, off, fill, col);
  DBM_CUDA(cudaGetLastError());
  return launch_csr_rows(off, 0, n, 2 * m, 2 * m, row, s);
}

// The rows [s0, s1) of the max-eps CSR only, from neighbour pairs that each have at least one
// endpoint in the batch (memory-bounded fit): entry positions are relative to off[s0], fill holds
// one cursor per batch row.
__global__ void csr_scatter_batch_kernel(const uint64_t* __restrict__ edges, int64_t cap,
                                         const unsigned long long* __restrict__ m_dev,
                                         const int64_t* __restrict__ off, int64_t s0, int64_t s1,
                                         int32_t* __restrict__ fill, uint32_t* __restrict__ col,
                                         int32_t* __restrict__ err)
{
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t m = static_cast<int64_t>(*m_dev) < cap ? static_cast<int64_t>(*m_dev) : cap;
  const bool valid = q < m;
  const uint64_t w = valid ? edges[q] : 0;
  const uint32_t i = static_cast<uint32_t>(w >> 32);
  const uint32_t lo = static_cast<uint32_t>(w);
  const uint32_t j = lo & kColMask;
  const uint32_t code = lo & ~kColMask;
  const bool own_i = valid && i >= s0 && i < s1, own_j = valid && j >= s0 && j < s1;
  const int32_t ki = warp_claim(fill, own_i ? static_cast<uint32_t>(i - s0) : kNoRow);
  const int32_t kj = warp_claim(fill, own_j ? static_cast<uint32_t>(j - s0) : kNoRow);
  if (!valid) return;
  const int64_t base = off[s0];
  // a row never receives more entries than its degree (same pairs as the degree pass); the
  // checks keep every write inside the buffers all the same and report a violation
  if (own_i) {
    const int64_t qi = off[i] - base + ki;
    if (qi < off[i + 1] - base && qi < cap) {
      col[qi] = code | j;
    } else {
      atomicOr(err, kErrGraphMismatch);
    }
  }
  if (own_j) {
    const int64_t qj = off[j] - base + kj;
    if (qj < off[j + 1] - base && qj < cap) {
      col[qj] = code | i;
    } else {
      atomicOr(err, kErrGraphMismatch);
    }
  }
}

// m_dev: the number of pairs (the distance pass's cursor, read on the device), at most cap.
Status launch_csr_scatter_batch(const uint64_t* edges, int64_t cap, const unsigned long long* m_dev, const int64_t* off,
                                int64_t s0, int64_t s1, int32_t* fill, uint32_t* col, int32_t* row, int32_t* err,
                                cudaStream_t s)
{
  if (cap <= 0) return Status::Ok();
  count_launch();
  csr_scatter_batch_kernel<<<static_cast<unsigned>(ceil_div(cap, 256)), 256, 0, s>>>(edges, cap, m_dev, off, s0, s1,
                                                                                     fill, col, err);
  DBM_CUDA(cudaGetLastError());
  return launch_csr_rows(off, s0, s1, cap, cap, row, s);
}

// ---- the tile pairs of one row batch (memory-bounded fit) ----------------------------------
// flags[q] = 1 iff worklist entry q (J << 32 | I) has tile I or tile J in [t0, t1)
__global__ void work_flags_kernel(const long long* __restrict__ work, int64_t count, int64_t t0, int64_t t1,
                                  int32_t* __restrict__ flags)
{
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= count) return;
  const long long e = work[q];
  const int64_t I = e & 0xffffffffLL, J = e >> 32;
  flags[q] = ((I >= t0 && I < t1) || (J >= t0 && J < t1)) ? 1 : 0;
}

// order-preserving compaction: out[pos[q]] = work[q] for flagged q
__global__ void work_compact_kernel(const long long* __restrict__ work, int64_t count,
                                    const int32_t* __restrict__ flags, const int64_t* __restrict__ pos,
                                    long long* __restrict__ out)
{
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= count) return;
  if (flags[q]) out[pos[q]] = work[q];
}

// The worklist entries touching tiles [t0, t1), in worklist order; *pos_out + count is the
// device word holding their number.
Status launch_batch_worklist(const long long* work, int64_t count, int64_t t0, int64_t t1, int32_t* flags,
                             int64_t* pos, void* scan_scratch, size_t scan_bytes, long long* out, cudaStream_t s)
{
  if (count <= 0) {
    DBM_CUDA(cudaMemsetAsync(pos, 0, sizeof(int64_t), s));
    return Status::Ok();
  }
  count_launch();
  work_flags_kernel<<<static_cast<unsigned>(ceil_div(count, 256)), 256, 0, s>>>(work, count, t0, t1, flags);
  DBM_CUDA(cudaGetLastError());
  DBM_TRY(exclusive_scan_i32(flags, pos, count, scan_scratch, scan_bytes, s));
  count_launch();
  work_compact_kernel<<<static_cast<unsigned>(ceil_div(count, 256)), 256, 0, s>>>(work, count, flags, pos, out);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// per-batch nnz at the largest eps, self pairs included (the reference's vd[n_points])
__global__ void batch_nnz_kernel(const int64_t* __restrict__ off, int64_t n, int64_t bs, int64_t nb,
                                 int64_t* __restrict__ out)
{
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const int64_t s0 = b * bs;
  const int64_t t0 = (s0 + bs < n) ? (s0 + bs) : n;
  out[b] = off[t0] - off[s0] + (t0 - s0);
}

// out[e] = sum over rows of (deg[e][i] - 1): directed entries per eps without the self pairs
// (out zeroed by the caller)
__global__ void eps_totals_kernel(const int32_t* __restrict__ deg, int64_t n, int k,
                                  unsigned long long* __restrict__ out)
{
  __shared__ unsigned long long part[kMaxEps];
  if (threadIdx.x < kMaxEps) part[threadIdx.x] = 0;
  __syncthreads();
  for (int e = 0; e < k; ++e) {
    unsigned long long s = 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
      s += static_cast<unsigned long long>(deg[static_cast<int64_t>(e) * n + i] - 1);
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0 && s) atomicAdd(&part[e], s);
  }
  __syncthreads();
  if (threadIdx.x < k && part[threadIdx.x]) atomicAdd(out + threadIdx.x, part[threadIdx.x]);
}

Status launch_eps_totals(const int32_t* deg, int64_t n, int k, unsigned long long* out, int sm_count, cudaStream_t s)
{
  DBM_CUDA(cudaMemsetAsync(out, 0, sizeof(unsigned long long) * k, s));
  count_launch();
  const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), sm_count * 4)));
  eps_totals_kernel<<<blocks, 256, 0, s>>>(deg, n, k, out);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

Status launch_batch_nnz(const int64_t* off, int64_t n, int64_t bs, int64_t nb, int64_t* out,
                        cudaStream_t s)
{
  count_launch();
  batch_nnz_kernel<<<static_cast<unsigned>(ceil_div(nb, 256)), 256, 0, s>>>(off, n, bs, nb, out);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// ---- all smaller eps of a batch at once (annotated route) -------------------------------------
// counts[e*rows + r] = deg[e][s0 + r] - 1, e < ne (= k - 1)
__global__ void slab_counts_all_kernel(const int32_t* __restrict__ deg, int64_t n, int ne, int64_t s0,
                                       int64_t rows, int32_t* __restrict__ counts)
{
  const int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (x >= rows * ne) return;
  const int64_t e = x / rows, r = x - e * rows;
  counts[x] = deg[e * n + s0 + r] - 1;
}

// One warp per batch row: one pass over its max-eps entries writes every smaller-eps slab e
// (entries with code <= e), order-preserving, at off_flat[e*rows + r].  Entry q of the max-eps
// CSR is col[q - col_base] (col_base = off[s0] when col holds only this batch's rows).
__global__ void filter_all_kernel(const int64_t* __restrict__ off, const uint32_t* __restrict__ col, int64_t col_base,
                                  int64_t s0, int64_t rows, int ne, const int64_t* __restrict__ off_flat,
                                  int32_t* __restrict__ col_flat, int32_t* __restrict__ row_flat)
{
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t r = s0 + warp;
  const int64_t beg = off[r], end = off[r + 1];
  const uint32_t below = (1u << lane) - 1u;
  // eps outermost with a scalar cursor (an array of cursors indexed by a runtime eps would live
  // in local memory); the row's entries are re-read from L1 for each eps
  for (int e = 0; e < ne; ++e) {
    int64_t out = off_flat[static_cast<int64_t>(e) * rows + warp];
    for (int64_t q0 = beg; q0 < end; q0 += 32) {
      const int64_t q = q0 + lane;
      uint32_t code = 0xffu, j = 0;
      if (q < end) {
        const uint32_t w = col[q - col_base];
        code = w >> kCodeShift;
        j = w & kColMask;
      }
      const bool keep = code <= static_cast<uint32_t>(e);
      const uint32_t bal = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const int64_t dst = out + __popc(bal & below);
        col_flat[dst] = static_cast<int32_t>(j);
        row_flat[dst] = static_cast<int32_t>(r);
      }
      out += __popc(bal);
    }
  }
}

Status launch_slab_counts_all(const int32_t* deg, int64_t n, int ne, int64_t s0, int64_t rows, int32_t* counts,
                              cudaStream_t s)
{
  if (ne <= 0 || rows <= 0) return Status::Ok();
  count_launch();
  slab_counts_all_kernel<<<static_cast<unsigned>(ceil_div(rows * ne, 256)), 256, 0, s>>>(deg, n, ne, s0, rows, counts);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

Status launch_filter_all(const int64_t* off, const uint32_t* col, int64_t col_base, int64_t s0, int64_t rows, int ne,
                         const int64_t* off_flat, int32_t* col_flat, int32_t* row_flat, cudaStream_t s)
{
  if (ne <= 0 || rows <= 0) return Status::Ok();
  count_launch();
  filter_all_kernel<<<static_cast<unsigned>(ceil_div(rows * 32, 256)), 256, 0, s>>>(off, col, col_base, s0, rows, ne,
                                                                                  off_flat, col_flat, row_flat);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// Label range check on the device (-1 <= label < n, src/main.cu:589-597): first bad position.
__global__ void label_range_kernel(const int32_t* __restrict__ labels, int64_t total, int64_t n,
                                   unsigned long long* __restrict__ first_bad)
{
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t v = labels[i];
    if (v < -1 || v >= n) atomicMin(first_bad, static_cast<unsigned long long>(i));
  }
}

Status launch_label_range(const int32_t* labels, int64_t total, int64_t n, unsigned long long* first_bad,
                          int sm_count, cudaStream_t s)
{
  count_launch();
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(total, 256), int64_t(sm_count) * 8));
  label_range_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(labels, total, n, first_bad);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// ---- core sample indices (sklearn convention) ---------------------------------------------------
__global__ void fill_i32_kernel(int32_t* __restrict__ p, int64_t count, int32_t v)
{
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

size_t core_indices_scratch_bytes(int64_t n)
{
  size_t temp = 0;
  thrust::counting_iterator<int32_t> it(0);
  cub::DeviceSelect::Flagged(nullptr, temp, it, static_cast<const uint8_t*>(nullptr), static_cast<int32_t*>(nullptr),
                             static_cast<int64_t*>(nullptr), static_cast<int>(n));
  return align_up(temp, 256) + 256;
}

// out[c*n ...] = ascending indices i with core[c*n + i] != 0, then -1
Status launch_core_indices(const uint8_t* core, int64_t n, int configs, int32_t* out, void* scratch,
                           size_t scratch_bytes, cudaStream_t s)
{
  if (scratch_bytes < core_indices_scratch_bytes(n)) return Status::Err(DBM_ERR_INVALID, "core index scratch too small");
  const int64_t total = n * configs;
  count_launch();
  fill_i32_kernel<<<static_cast<unsigned>(std::min<int64_t>(ceil_div(total, 256), 148 * 32)), 256, 0, s>>>(out, total, -1);
  DBM_CUDA(cudaGetLastError());
  int64_t* num = reinterpret_cast<int64_t*>(scratch);
  void* temp = static_cast<unsigned char*>(scratch) + 256;
  size_t temp_bytes = scratch_bytes - 256;
  thrust::counting_iterator<int32_t> it(0);
  for (int c = 0; c < configs; ++c) {
    count_launch();
    DBM_CUDA(cub::DeviceSelect::Flagged(temp, temp_bytes, it, core + static_cast<int64_t>(c) * n,
                                        out + static_cast<int64_t>(c) * n, num, static_cast<int>(n), s));
  }
  return Status::Ok();
}

}  // namespace dbm
