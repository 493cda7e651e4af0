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
constexpr int kDimBox = 64;          // dims per TMA box
constexpr uint32_t kWaitPolls = 1u << 24;

struct DistParams {
  int64_t n;
  int32_t d;
  int32_t k;
  int32_t dbox;                      // dims per box actually used (<= kDimBox)
  int32_t pad_;
  int64_t tile_pairs;                // T(T+1)/2
  unsigned long long* counters;      // [0] edge cursor, [1] next tile pair
  uint64_t* edges;
  uint64_t edge_cap;
  int32_t* hist;                     // k x n
  int32_t* err;
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

__global__ void __launch_bounds__(kDistThreads, 2)
dist_tri_kernel(const __grid_constant__ CUtensorMap xt_map, const DistParams p)
{
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  float* As = reinterpret_cast<float*>(dyn_smem);      // [dbox][128]
  float* Bs = As + static_cast<size_t>(p.dbox) * kTile;  // [dbox][128]
  __shared__ __align__(8) uint64_t bar;
  __shared__ long long s_tile;
  __shared__ float s_eps2[kMaxEps];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  if (tid < kMaxEps) s_eps2[tid] = p.eps2[tid];
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();

  const int64_t n = p.n;
  const float cutoff = p.eps2[p.k - 1];
  const uint32_t box_bytes = static_cast<uint32_t>(p.dbox) * kTile * sizeof(float);
  uint32_t phase = 0;
  const int lane = tid & 31;

  for (;;) {
    if (tid == 0) s_tile = static_cast<long long>(atomicAdd(p.counters + 1, 1ULL));
    __syncthreads();
    const long long c = s_tile;
    if (c >= p.tile_pairs) break;
    long long I, J;
    tri_coords(c, I, J);
    const int64_t row0 = I * kTile, col0 = J * kTile;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    for (int d0 = 0; d0 < p.d; d0 += p.dbox) {
      if (tid == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&bar, 2 * box_bytes);
        tma_load_2d(As, &xt_map, static_cast<int32_t>(row0), d0, &bar);
        tma_load_2d(Bs, &xt_map, static_cast<int32_t>(col0), d0, &bar);
      }
      const bool ok = mbar_wait_bounded(&bar, phase, kWaitPolls);
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicOr(p.err, kErrTmaTimeout);
        mbar_wait_bounded(&bar, phase, kWaitPolls);  // let the copy in flight land
        return;
      }
      phase ^= 1u;
      const int dk = min(p.dbox, p.d - d0);
#pragma unroll 2
      for (int t = 0; t < dk; ++t) {
        const float* arow = As + t * kTile;
        const float* brow = Bs + t * kTile;
        const float4 a0 = *reinterpret_cast<const float4*>(arow + ty * 4);
        const float4 a1 = *reinterpret_cast<const float4*>(arow + 64 + ty * 4);
        const float4 b0 = *reinterpret_cast<const float4*>(brow + tx * 4);
        const float4 b1 = *reinterpret_cast<const float4*>(brow + 64 + tx * 4);
        const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float diff = __fsub_rn(a[i], b[j]);
            acc[i][j] = __fmaf_rn(diff, diff, acc[i][j]);
          }
      }
      __syncthreads();  // all reads of this chunk done before the next TMA overwrites it
    }

    // ---- epilogue: neighbour pairs (i < j) within the largest eps --------------------
    const bool diag = (I == J);
    uint64_t nb = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t gi = row0 + ((i < 4) ? (ty * 4 + i) : (64 + ty * 4 + i - 4));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t gj = col0 + ((j < 4) ? (tx * 4 + j) : (64 + tx * 4 + j - 4));
        const bool v = (gi < n) && (gj < n) && (!diag || gj > gi) && (acc[i][j] <= cutoff);
        nb |= static_cast<uint64_t>(v) << (i * 8 + j);
      }
    }
    const int cnt = __popcll(nb);
    if (__any_sync(0xffffffffu, cnt != 0)) {
      int incl = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      unsigned long long base = 0;
      if (lane == 31) base = atomicAdd(p.counters, static_cast<unsigned long long>(total));
      base = __shfl_sync(0xffffffffu, base, 31);
      unsigned long long idx = base + static_cast<unsigned long long>(incl - cnt);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (!((nb >> (i * 8 + j)) & 1ull)) continue;
          const int64_t gi = row0 + ((i < 4) ? (ty * 4 + i) : (64 + ty * 4 + i - 4));
          const int64_t gj = col0 + ((j < 4) ? (tx * 4 + j) : (64 + tx * 4 + j - 4));
          const float v = acc[i][j];
          int code = 0;
          while (v > s_eps2[code]) ++code;  // terminates: v <= eps2[k-1]
          if (idx < p.edge_cap)
            p.edges[idx] = (static_cast<uint64_t>(gi) << 32) |
                           (static_cast<uint64_t>(code) << kCodeShift) | static_cast<uint64_t>(gj);
          ++idx;
          atomicAdd(p.hist + static_cast<int64_t>(code) * n + gi, 1);
          atomicAdd(p.hist + static_cast<int64_t>(code) * n + gj, 1);
        }
      }
    }
  }
}

// X (n x d, row-major) -> XT (dp x npad, dim-major), zero padded.
// Also flags NaN/Inf inputs, which the reference rejects before fitting (src/main.cu:1419-1423).
__global__ void transpose_pad_kernel(const float* __restrict__ x, float* __restrict__ xt, int64_t n,
                                     int32_t d, int32_t dp, int64_t npad, int32_t* __restrict__ err)
{
  __shared__ float tile[32][33];
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int32_t t0 = static_cast<int32_t>(blockIdx.y) * 32;
  bool bad = false;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t i = i0 + r;
    const int32_t t = t0 + static_cast<int32_t>(threadIdx.x);
    const float v = (i < n && t < d) ? x[i * d + t] : 0.0f;
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

Status transpose_pad(const float* x, float* xt, int64_t n, int32_t d, int32_t* err, cudaStream_t s)
{
  const int32_t dp = padded_dims(d);
  const int64_t npad = padded_points(n);
  dim3 grid(static_cast<unsigned>(ceil_div(npad, 32)), static_cast<unsigned>(ceil_div(dp, 32)));
  count_launch();
  transpose_pad_kernel<<<grid, dim3(32, 8), 0, s>>>(x, xt, n, d, dp, npad, err);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}


Status launch_distance(const DistLaunch& a, cudaStream_t s)
{
  auto encode = get_encode_fn();
  if (!encode) return Status::Err(DBM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int32_t dp = padded_dims(a.d);
  const int64_t npad = padded_points(a.n);
  const int32_t dbox = dp < kDimBox ? dp : kDimBox;

  CUtensorMap map;
  const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(a.n), static_cast<cuuint64_t>(dp)};
  const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(npad) * sizeof(float)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTile), static_cast<cuuint32_t>(dbox)};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.xt), gdim,
                      gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return Status::Err(DBM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");

  DistParams p{};
  p.n = a.n;
  p.d = a.d;
  p.k = a.k;
  p.dbox = dbox;
  const int64_t T = ceil_div(a.n, kTile);
  p.tile_pairs = T * (T + 1) / 2;
  p.counters = a.counters;
  p.edges = a.edges;
  p.edge_cap = a.edge_cap;
  p.hist = a.hist;
  p.err = a.err;
  for (int e = 0; e < kMaxEps; ++e) p.eps2[e] = e < a.k ? a.eps2[e] : a.eps2[a.k - 1];

  const size_t smem = 2ull * dbox * kTile * sizeof(float);
  DBM_CUDA(cudaFuncSetAttribute(dist_tri_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  int per_sm = 0;
  DBM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dist_tri_kernel, kDistThreads,
                                                         smem));
  if (per_sm < 1) per_sm = 1;
  int64_t grid = static_cast<int64_t>(a.sm_count) * per_sm;
  if (grid > p.tile_pairs) grid = p.tile_pairs;
  count_launch();
  dist_tri_kernel<<<static_cast<unsigned>(grid), kDistThreads, smem, s>>>(map, p);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

}  // namespace dbm
