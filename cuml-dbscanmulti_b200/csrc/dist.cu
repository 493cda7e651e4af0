// dist.cu -- multi-eps neighbourhood kernel: fp32 L2 over the upper triangle of pair tiles.
//
// Replaces the reference's per-row search kernels (src/multi/eps_neighborhood.cuh:97-347,
// epsNeighborhoodReg/Generic/GlobalKernel) and the cuVS eps-search they stand in for.
// Arithmetic per pair is the reference's, bit for bit: acc = fma(q[t]-p[t], q[t]-p[t], acc)
// for t = 0..D-1 in order, code = smallest e with acc <= eps2[e] (255 = none)
// (eps_neighborhood.cuh:151-168).  Because that value is bitwise symmetric in (i, j)
// ((q-p)^2 == (p-q)^2 exactly), each unordered pair is evaluated once: CTAs walk the tile
// pairs (I <= J) of the N x N grid, and every neighbour pair found is credited to both rows.
//
// Layout: X is first copied into XT, a dim-major [Dp][Npad] float32 array (Dp = D rounded up
// to 4, Npad = N rounded up to 4) so that a 128-point tile of one dimension is a contiguous
// 512-byte row; one 2-D TMA box {128 points, up to 64 dims} lands as smem[dim][point], which
// the 16x16 thread grid reads with conflict-free 16-byte loads.  Each thread owns 8 rows x 8
// columns of the 128 x 128 tile and keeps the 64 FMA chains in registers.
//
// Outputs per launch:
//   hist[c*N + i]  number of pairs (i, j != i) whose code is c (atomic, exact),
//   edges[]        one 64-bit word per neighbour pair i < j: i << 32 | code << 28 | j,
//                  appended with warp-aggregated atomics up to `edge_cap` (the cursor keeps
//                  counting past it so the host learns the exact size),
//   err            bit flags (bounded TMA wait ran out).
#include "dbm_internal.cuh"

#include <cudaTypedefs.h>

#include <cmath>

namespace dbm {

constexpr int kTile = 128;
constexpr int kDistThreads = 256;
// dims per TMA box: 32 keeps a CTA's two stages at 64 KB, so two CTAs share an SM (the 64-dim
// boxes of 128 KB allowed one: calibrated dense C5 at N = 100,000, exact-kernel time 49.9 -> 43.0 ms)
constexpr int kDimBox = 32;
constexpr uint32_t kWaitPolls = 1u << 24;
#ifndef DBM_PROBE_DIMS
#define DBM_PROBE_DIMS 8
#endif
constexpr int kProbeDims = DBM_PROBE_DIMS;  // dims between two early-exit checks


struct DistParams {
  int64_t n;
  int32_t d;
  int32_t k;
  int32_t dbox;                      // dims per box actually used (<= kDimBox)
  int32_t nchunks;                   // ceil(d / dbox)
  int32_t shard, nshards;            // this launch's share of the work items (tile pairs, or
  int64_t item_count;                // worklist entries): item_count of them, mapped by shard_item
  const long long* work;             // worklist of tile-pair indices (nullptr: item = tile pair)
  const unsigned long long* count_dev;  // when set, item_count is read here on the device
  unsigned long long* counters;      // [0] edge cursor, [1] next tile pair
  uint64_t* edges;
  uint64_t edge_cap;
  int32_t* hist;                     // k x n
  int32_t* err;
  const float* xt;                   // dp x npad (for re-evaluating neighbour pairs)
  int64_t npad;
  const int32_t* perm;               // original index of each XT column (nullptr: identity)
  int64_t keep_lo, keep_hi;          // emit only pairs with an endpoint in [keep_lo, keep_hi)
  float eps2[kMaxEps];
};

// (I, J) with I <= J from the column-major index c of the upper triangle.
__device__ __forceinline__ void tri_coords(long long c, long long& I, long long& J)
{
  long long j = static_cast<long long>((sqrt(8.0 * static_cast<double>(c) + 1.0) - 1.0) * 0.5);
  while (j * (j + 1) / 2 > c) --j;
  while ((j + 1) * (j + 2) / 2 <= c) ++j;
  J = j;
  I = c - j * (j + 1) / 2;
}

// A work item: a worklist entry (J << 32 | I) or, without a worklist, a tile-pair index.
__device__ __forceinline__ void item_coords(const DistParams& p, long long e, long long& I, long long& J)
{
  if (p.work) {
    I = e & 0xffffffffLL;
    J = e >> 32;
  } else {
    tri_coords(e, I, J);
  }
}

// ---- packed fp32 pairs (sm_100: .f32x2, each lane rounded exactly like the scalar op) ----------
__device__ __forceinline__ uint64_t pack2(float lo, float hi)
{
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi)
{
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b)
{
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sqacc2(uint64_t diff, uint64_t acc)
{
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %1, %2;" : "=l"(d) : "l"(diff), "l"(acc));
  return d;
}

// Shared-memory plan per CTA: two stages of {A tile, B tile}, each [dbox][128] floats.
__host__ __device__ constexpr size_t dist_smem_bytes(int dbox)
{
  return static_cast<size_t>(dbox) * kTile * sizeof(float) * 4;
}

// MinBlocks: CTAs per SM the register budget is sized for (2 when the tile buffers let two CTAs
// share an SM, 1 for the 64-dim boxes, whose 128 KB of buffers admit only one anyway).
template <int MinBlocks>
__global__ void __launch_bounds__(kDistThreads, MinBlocks)
dist_tri_kernel(const __grid_constant__ CUtensorMap xt_map, const DistParams p)
{
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  const int box_floats = p.dbox * kTile;
  float* As0 = reinterpret_cast<float*>(dyn_smem);
  float* Bs0 = As0 + box_floats;
  float* As1 = Bs0 + box_floats;
  float* Bs1 = As1 + box_floats;
  // per-(code, local row) pair counts of the current tile pair: rows of tile I at [0, 128), of
  // tile J at [128, 256); flushed to hist once per tile pair (a dense tile pair has up to 16,384
  // neighbour pairs, i.e. 32,768 global atomics otherwise)
  int32_t* s_hist = reinterpret_cast<int32_t*>(Bs1 + box_floats);
  __shared__ __align__(8) uint64_t full[2];
  __shared__ long long s_tile[2];  // tile pair index held by each stage (< 0: none)
  __shared__ float s_eps2[kMaxEps];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int lane = tid & 31;
  if (tid < kMaxEps) s_eps2[tid] = p.eps2[tid];
  if (p.hist)
    for (int q = tid; q < p.k * 2 * kTile; q += kDistThreads) s_hist[q] = 0;
  const uint32_t box_bytes = static_cast<uint32_t>(box_floats) * sizeof(float);

  auto next_tile = [&]() -> long long {
    const long long i = static_cast<long long>(atomicAdd(p.counters + 1, 1ULL));
    const long long limit = p.count_dev ? static_cast<long long>(*p.count_dev) : p.item_count;
    if (i >= limit) return -1;
    const long long g = shard_item(i, p.shard, p.nshards);
    return p.work ? p.work[g] : g;
  };
  auto issue = [&](int stage, long long tile, int chunk) {
    // one thread: record the item and start both tile loads of this stage
    s_tile[stage] = tile;
    if (tile < 0) return;
    long long I, J;
    item_coords(p, tile, I, J);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&full[stage], 2 * box_bytes);
    float* a = stage ? As1 : As0;
    float* b = stage ? Bs1 : Bs0;
    tma_load_2d(a, &xt_map, static_cast<int32_t>(I * kTile), chunk * p.dbox, &full[stage]);
    tma_load_2d(b, &xt_map, static_cast<int32_t>(J * kTile), chunk * p.dbox, &full[stage]);
  };

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_fence_init();
    issue(0, next_tile(), 0);
  }
  __syncthreads();

  const int64_t n = p.n;
  const float cutoff = p.eps2[p.k - 1];
  uint32_t phase[2] = {0u, 0u};
  int stage = 0, chunk = 0;
  uint64_t acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0ull;

  bool warp_done = false;      // this warp's pairs of the current tile are all beyond the cutoff
  long long dims_done = 0;     // dims this warp evaluated, over all its tiles
  for (;;) {
    const long long c = s_tile[stage];
    if (c < 0) break;
    bool warp_hits = false;     // this warp found neighbour pairs in the tile pair's epilogue
    if (chunk == 0) warp_done = false;
    const bool ok = mbar_wait_bounded(&full[stage], phase[stage], kWaitPolls);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(p.err, kErrTmaTimeout);
      mbar_wait_bounded(&full[stage], phase[stage], kWaitPolls);
      mbar_wait_bounded(&full[stage ^ 1], phase[stage ^ 1], kWaitPolls);
      return;
    }
    phase[stage] ^= 1u;
    const bool last_chunk = (chunk + 1 == p.nchunks);
    if (tid == 0) {
      // prefetch the next item into the other stage (released by the previous iteration)
      if (!last_chunk)
        issue(stage ^ 1, c, chunk + 1);
      else
        issue(stage ^ 1, next_tile(), 0);
    }
    const float* As = stage ? As1 : As0;
    const float* Bs = stage ? Bs1 : Bs0;
    const int dk = min(p.dbox, p.d - chunk * p.dbox);
    // Early exit, result-neutral: partial sums never decrease along the dims (fma(d, d, acc)
    // >= acc in round-to-nearest), so once every pair this warp holds is above the largest
    // eps^2 no code can change; the warp skips the remaining dims of the tile (the reference's
    // generic kernel breaks the same way per pair, eps_neighborhood.cuh:247).
    auto step = [&](int t) {
      uint64_t a[8];
      // (a, a) operand pairs for the 8 rows; (b, b') pairs come straight from 16-byte loads
      const float4 f0 = *reinterpret_cast<const float4*>(As + t * kTile + ty * 4);
      const float4 f1 = *reinterpret_cast<const float4*>(As + t * kTile + 64 + ty * 4);
      a[0] = pack2(f0.x, f0.x); a[1] = pack2(f0.y, f0.y); a[2] = pack2(f0.z, f0.z); a[3] = pack2(f0.w, f0.w);
      a[4] = pack2(f1.x, f1.x); a[5] = pack2(f1.y, f1.y); a[6] = pack2(f1.z, f1.z); a[7] = pack2(f1.w, f1.w);
      const ulonglong2 b01 = *reinterpret_cast<const ulonglong2*>(Bs + t * kTile + tx * 4);
      const ulonglong2 b23 = *reinterpret_cast<const ulonglong2*>(Bs + t * kTile + 64 + tx * 4);
      const uint64_t b[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = sqacc2(sub2(a[i], b[j]), acc[i][j]);
    };
    for (int t0 = 0; t0 < dk && !warp_done; t0 += kProbeDims) {
      const int tn = min(kProbeDims, dk - t0);
      if (tn == kProbeDims) {
#pragma unroll
        for (int u = 0; u < kProbeDims; ++u) step(t0 + u);
      } else {
        for (int u = 0; u < tn; ++u) step(t0 + u);
      }
      dims_done += tn;
      if (t0 + tn < dk || !last_chunk) {
        float mn = INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float lo, hi;
            unpack2(acc[i][j], lo, hi);
            mn = fminf(mn, fminf(lo, hi));
          }
        warp_done = __all_sync(0xffffffffu, mn > cutoff);
      }
    }

    if (last_chunk) {
      // ---- epilogue: neighbour pairs (i < j) within the largest eps -------------------
      // Fast path: nothing to do unless some pair of the warp is within the cutoff.
      float mn = INFINITY;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float lo, hi;
          unpack2(acc[i][j], lo, hi);
          mn = fminf(mn, fminf(lo, hi));
        }
      if (__any_sync(0xffffffffu, mn <= cutoff)) {
        long long I, J;
        item_coords(p, c, I, J);
        const int32_t row0 = static_cast<int32_t>(I) * kTile, col0 = static_cast<int32_t>(J) * kTile;
        const int32_t n32 = static_cast<int32_t>(n);
        const bool diag = (I == J);
        uint64_t nb = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int32_t gi = row0 + ((i < 4) ? (ty * 4 + i) : (64 + ty * 4 + i - 4));
#pragma unroll
          for (int jp = 0; jp < 4; ++jp) {
            float w[2];
            unpack2(acc[i][jp], w[0], w[1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int j = 2 * jp + h;
              const int32_t gj = col0 + ((j < 4) ? (tx * 4 + j) : (64 + tx * 4 + j - 4));
              const bool hit = (gi < n32) && (gj < n32) && (!diag || gj > gi) && (w[h] <= cutoff) &&
                               keep_pair(gi, gj, p.keep_lo, p.keep_hi);
              nb |= static_cast<uint64_t>(hit) << (i * 8 + j);
            }
          }
        }
        const int cnt = __popcll(nb);
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += u;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        unsigned long long base = 0;
        if (lane == 31 && total > 0) base = atomicAdd(p.counters, static_cast<unsigned long long>(total));
        base = __shfl_sync(0xffffffffu, base, 31);
        unsigned long long idx = base + static_cast<unsigned long long>(incl - cnt);
        // Codes straight from the accumulators: each lane of acc[i][jp] is the reference's
        // sequential fp32 chain of its pair over all D dims (per-lane IEEE rounding of
        // sub.rn.f32x2 / fma.rn.f32x2, dims in order, across chunks); the loops are unrolled so
        // the accumulators stay in registers.
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int lr = (i < 4) ? (ty * 4 + i) : (64 + ty * 4 + i - 4);
#pragma unroll
          for (int jp = 0; jp < 4; ++jp) {
            float w[2];
            unpack2(acc[i][jp], w[0], w[1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int j = 2 * jp + h;
              if (!((nb >> (i * 8 + j)) & 1ull)) continue;
              const int lc = (j < 4) ? (tx * 4 + j) : (64 + tx * 4 + j - 4);
              const int32_t gi = row0 + lr, gj = col0 + lc;
              int code = 0;
              while (w[h] > s_eps2[code]) ++code;  // terminates: w <= eps2[k-1]
              int32_t oi = gi, oj = gj;  // original point indices
              if (p.perm) {
                oi = p.perm[gi];
                oj = p.perm[gj];
              }
              const int32_t lo = min(oi, oj), hi = max(oi, oj);
              if (idx < p.edge_cap)
                p.edges[idx] = (static_cast<uint64_t>(lo) << 32) |
                               (static_cast<uint64_t>(code) << kCodeShift) | static_cast<uint64_t>(hi);
              ++idx;
              if (p.hist) {
                atomicAdd(s_hist + code * 2 * kTile + lr, 1);
                atomicAdd(s_hist + code * 2 * kTile + kTile + lc, 1);
              }
            }
          }
        }
        warp_hits = true;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0ull;
    }
    // this stage's buffers are free; the next item's descriptor is visible; the tile pair's counts
    // are complete
    const bool flush = __syncthreads_or(warp_hits) && p.hist;
    if (flush) {
      // thread r owns local row r: tile I's rows below 128, tile J's from 128
      long long I, J;
      item_coords(p, c, I, J);
      const int32_t g = tid < kTile ? static_cast<int32_t>(I) * kTile + tid : static_cast<int32_t>(J) * kTile + tid - kTile;
      for (int e = 0; e < p.k; ++e) {
        const int32_t v = s_hist[e * 2 * kTile + tid];
        if (v) {
          atomicAdd(p.hist + static_cast<int64_t>(e) * n + (p.perm ? p.perm[g] : g), v);
          s_hist[e * 2 * kTile + tid] = 0;
        }
      }
      __syncthreads();  // cleared before the next tile pair counts
    }
    stage ^= 1;
    chunk = last_chunk ? 0 : chunk + 1;
  }
  if (lane == 0 && dims_done) atomicAdd(p.counters + 2, static_cast<unsigned long long>(dims_done));
}

// X (n x d, row-major) -> XT (rows x npad, dim-major), zero padded (rows >= d).
// Also flags NaN/Inf inputs, which the reference rejects before fitting (src/main.cu:1419-1423).
__global__ void transpose_pad_kernel(const float* __restrict__ x, float* __restrict__ xt, int64_t n,
                                     int32_t d, int32_t dp, int64_t npad, int32_t* __restrict__ err,
                                     const int32_t* __restrict__ perm)
{
  __shared__ float tile[32][33];
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int32_t t0 = static_cast<int32_t>(blockIdx.y) * 32;
  bool bad = false;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t i = i0 + r;
    const int32_t t = t0 + static_cast<int32_t>(threadIdx.x);
    const int64_t src = (perm && i < n) ? static_cast<int64_t>(perm[i]) : i;
    const float v = (i < n && t < d) ? x[src * d + t] : 0.0f;
    bad |= !isfinite(v);
    tile[r][threadIdx.x] = v;
  }
  if (bad) atomicOr(err, kErrNonFinite);
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int32_t t = t0 + r;
    const int64_t i = i0 + threadIdx.x;
    if (t < dp && i < npad) xt[static_cast<int64_t>(t) * npad + i] = tile[threadIdx.x][r];
  }
}

// The same for d <= kTransposeMaxD: PTS points per block and every row of them at once, so each
// point's row is gathered once (one contiguous 4d-byte read, eight loads in flight per thread)
// and every XT row is written as 4 PTS-byte runs.  Shared pitch d or d + 1, whichever is odd
// (conflict-free column reads).  With PTS = 128 a block is one 128-point tile and, given lo / hi,
// also writes the tile's box (min / max of each dim over its points < n, dim-major
// lo[t * tiles + tile]: what tile_box_kernel computes from XT) while the tile is in shared memory.
constexpr int kTransposeMaxD = 128;
constexpr int kTransposeBoxMaxD = 64;  // 128 x 65 floats: the fused box variant stays within 48 KB
template <int PTS>
__global__ void __launch_bounds__(256) transpose_rows_kernel(const float* __restrict__ x, float* __restrict__ xt,
                                                             int64_t n, int32_t d, int32_t dp, int64_t npad,
                                                             int32_t* __restrict__ err, const int32_t* __restrict__ perm,
                                                             float* __restrict__ lo, float* __restrict__ hi)
{
  extern __shared__ float tile[];  // [PTS][pitch]
  __shared__ int32_t src[PTS];
  const int pitch = d | 1;
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * PTS;
  if (threadIdx.x < PTS) {
    const int64_t i = i0 + threadIdx.x;
    src[threadIdx.x] = i < n ? (perm ? perm[i] : static_cast<int32_t>(i)) : -1;
  }
  __syncthreads();
  bool bad = false;
  const int total = PTS * d;
  constexpr int kInFlight = 8;
  for (int base = threadIdx.x; base < total; base += kInFlight * 256) {
    float v[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int idx = base + u * 256;
      v[u] = 0.0f;
      if (idx < total) {
        const int r = idx / d, t = idx - r * d;
        const int32_t sr = src[r];
        if (sr >= 0) v[u] = x[static_cast<int64_t>(sr) * d + t];
      }
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int idx = base + u * 256;
      if (idx < total) {
        const int r = idx / d, t = idx - r * d;
        bad |= !isfinite(v[u]);
        tile[r * pitch + t] = v[u];
      }
    }
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(err, kErrNonFinite);
  for (int idx = threadIdx.x; idx < dp * PTS; idx += blockDim.x) {
    const int t = idx / PTS, r = idx - t * PTS;
    const int64_t i = i0 + r;
    if (i < npad) xt[static_cast<int64_t>(t) * npad + i] = t < d ? tile[r * pitch + t] : 0.0f;
  }
  if (PTS == 128 && lo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int valid = n - i0 < PTS ? static_cast<int>(n - i0) : PTS;
    const int64_t tiles = gridDim.x;
    for (int t = warp; t < d; t += 8) {
      float mn = INFINITY, mx = -INFINITY;
      for (int r = lane; r < valid; r += 32) {
        const float v = tile[r * pitch + t];
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      }
      if (lane == 0) {
        lo[static_cast<int64_t>(t) * tiles + blockIdx.x] = mn;
        hi[static_cast<int64_t>(t) * tiles + blockIdx.x] = mx;
      }
    }
  }
}

// ---- host side ------------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn()
{
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
          cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

int32_t padded_dims(int32_t d) { return (d + 3) / 4 * 4; }
int64_t padded_points(int64_t n) { return (n + 3) / 4 * 4; }

Status launch_tile_boxes(const float* xt, int64_t n, int64_t npad, int32_t d, float* lo, float* hi, cudaStream_t s);

Status transpose_pad(const float* x, float* xt, int64_t n, int32_t d, int32_t* err, cudaStream_t s,
                     const int32_t* perm, int32_t rows, float* box_lo, float* box_hi)
{
  const int32_t dp = rows > padded_dims(d) ? rows : padded_dims(d);
  const int64_t npad = padded_points(n);
  count_launch();
  if (d <= kTransposeBoxMaxD) {
    // one block per 128-point tile (npad <= 128 * tiles), boxes written on the way when asked
    const size_t smem = sizeof(float) * 128 * static_cast<size_t>(d | 1);
    transpose_rows_kernel<128><<<static_cast<unsigned>(ceil_div(npad, 128)), 256, smem, s>>>(
      x, xt, n, d, dp, npad, err, perm, box_lo, box_hi);
    DBM_CUDA(cudaGetLastError());
    return Status::Ok();
  }
  if (d <= kTransposeMaxD) {
    const size_t smem = sizeof(float) * 64 * static_cast<size_t>(d | 1);
    transpose_rows_kernel<64><<<static_cast<unsigned>(ceil_div(npad, 64)), 256, smem, s>>>(x, xt, n, d, dp, npad, err,
                                                                                           perm, nullptr, nullptr);
  } else {
    dim3 grid(static_cast<unsigned>(ceil_div(npad, 32)), static_cast<unsigned>(ceil_div(dp, 32)));
    transpose_pad_kernel<<<grid, dim3(32, 8), 0, s>>>(x, xt, n, d, dp, npad, err, perm);
  }
  DBM_CUDA(cudaGetLastError());
  if (box_lo) return launch_tile_boxes(xt, n, npad, d, box_lo, box_hi, s);
  return Status::Ok();
}


// Tensor map over XT (dp x npad fp32, dim-major): boxes of {128 points, dbox dims}.
Status make_tile_map(const float* xt, int64_t n, int32_t rows, CUtensorMap* map)
{
  auto encode = get_encode_fn();
  if (!encode) return Status::Err(DBM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (rows < 1 || rows > 256) return Status::Err(DBM_ERR_INVALID, "tile map rows out of range");
  const int64_t npad = padded_points(n);
  const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(rows)};
  const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(npad) * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTile), static_cast<cuuint32_t>(rows)};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(xt), gdim, gstride, box,
                      estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return Status::Err(DBM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return Status::Ok();
}

Status make_xt_map(const float* xt, int64_t n, int32_t d, CUtensorMap* map, int32_t* dbox_out)
{
  auto encode = get_encode_fn();
  if (!encode) return Status::Err(DBM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int32_t dp = padded_dims(d);
  const int64_t npad = padded_points(n);
  const int32_t dbox = dp < kDimBox ? dp : kDimBox;
  const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(dp)};
  const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(npad) * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTile), static_cast<cuuint32_t>(dbox)};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(xt), gdim, gstride, box,
                      estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return Status::Err(DBM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  *dbox_out = dbox;
  return Status::Ok();
}

Status launch_distance(const DistLaunch& a, cudaStream_t s)
{
  const int64_t npad = padded_points(a.n);
  CUtensorMap map;
  int32_t dbox = 0;
  DBM_TRY(make_xt_map(a.xt, a.n, a.d, &map, &dbox));

  DistParams p{};
  p.n = a.n;
  p.d = a.d;
  p.k = a.k;
  p.dbox = dbox;
  p.nchunks = static_cast<int32_t>(ceil_div(a.d, dbox));
  const int64_t T = ceil_div(a.n, kTile);
  const int64_t items = a.work ? a.work_count : T * (T + 1) / 2;
  const int shards = a.nshards > 0 ? a.nshards : 1;
  p.shard = a.shard;
  p.nshards = shards;
  p.item_count = shard_items(items, a.shard, shards);
  p.work = a.work;
  p.count_dev = a.work_count_dev;
  if (a.work_count_dev) {  // a list of this launch's own (the screen's fallback tile pairs)
    p.shard = 0;
    p.nshards = 1;
    p.item_count = 0;
  }
  p.counters = a.counters;
  p.edges = a.edges;
  p.edge_cap = a.edge_cap;
  p.hist = a.hist;
  p.err = a.err;
  p.xt = a.xt;
  p.npad = npad;
  p.perm = a.perm;
  p.keep_lo = a.keep_lo;
  p.keep_hi = a.keep_hi;
  for (int e = 0; e < kMaxEps; ++e) p.eps2[e] = e < a.k ? a.eps2[e] : a.eps2[a.k - 1];

  const size_t smem = dist_smem_bytes(dbox) + (a.hist ? sizeof(int32_t) * a.k * 2 * kTile : 0);
  const bool one_per_sm = smem > 100 * 1024;
  auto kernel = one_per_sm ? dist_tri_kernel<1> : dist_tri_kernel<2>;
  DBM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  int per_sm = 0;
  DBM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kDistThreads, smem));
  if (per_sm < 1) per_sm = 1;
  int64_t grid = static_cast<int64_t>(a.sm_count) * per_sm;
  if (!a.work_count_dev && grid > p.item_count) grid = p.item_count;
  if (grid < 1) return Status::Ok();
  count_launch();
  kernel<<<static_cast<unsigned>(grid), kDistThreads, smem, s>>>(map, p);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

}  // namespace dbm
