// order.cu -- spatial ordering of the points before the distance pass.
//
// The distance kernel stops a warp as soon as every pair it holds is beyond the largest eps
// (partial sums only grow along the dims).  That pays only if the 128 points of a tile are
// close to each other in their leading coordinates, so the points are visited in Z-order
// (Morton order) of their first m <= 4 coordinates: a tile then covers a small region of
// those coordinates and most tile pairs are separated after the first few dims.
//
// Nothing about the results depends on the order: the distance of a pair is the same float
// whichever point comes first, and the kernel writes every neighbour pair and every degree
// back under the original indices (perm[]), so labels, degrees and core masks are identical.
#include "dbm_internal.cuh"

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>

namespace dbm {

// float <-> unsigned key that preserves order (for atomic min/max on floats)
__device__ __forceinline__ uint32_t float_to_ordered(float f)
{
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(uint32_t u)
{
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// lohi[2t] = ordered(min over points of x[t]), lohi[2t+1] = ordered(max), t < m
__global__ void bbox_kernel(const float* __restrict__ x, int64_t n, int32_t d, int m,
                            uint32_t* __restrict__ lohi)
{
  __shared__ uint32_t smin[4], smax[4];
  if (threadIdx.x < 4) {
    smin[threadIdx.x] = 0xffffffffu;
    smax[threadIdx.x] = 0u;
  }
  __syncthreads();
  uint32_t lo[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu}, hi[4] = {0, 0, 0, 0};
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    for (int t = 0; t < m; ++t) {
      const uint32_t v = float_to_ordered(x[i * d + t]);
      lo[t] = min(lo[t], v);
      hi[t] = max(hi[t], v);
    }
  }
  for (int t = 0; t < m; ++t) {
    atomicMin(&smin[t], lo[t]);
    atomicMax(&smax[t], hi[t]);
  }
  __syncthreads();
  if (threadIdx.x < m) {
    atomicMin(&lohi[2 * threadIdx.x], smin[threadIdx.x]);
    atomicMax(&lohi[2 * threadIdx.x + 1], smax[threadIdx.x]);
  }
}

__global__ void bbox_init_kernel(uint32_t* lohi)
{
  if (threadIdx.x < 8) lohi[threadIdx.x] = (threadIdx.x & 1) ? 0u : 0xffffffffu;
}

// key = bit-interleave of the first m coordinates quantised to min(32/m, 24) bits each; val = index
__global__ void morton_kernel(const float* __restrict__ x, int64_t n, int32_t d, int m,
                              const uint32_t* __restrict__ lohi, uint32_t* __restrict__ key,
                              int32_t* __restrict__ val)
{
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int bits = min(32 / m, 24);  // <= 24: finer steps are below float resolution anyway
  const float levels = ldexpf(1.0f, bits);
  uint32_t q[4] = {0, 0, 0, 0};
  for (int t = 0; t < m; ++t) {
    const float lo = ordered_to_float(lohi[2 * t]), hi = ordered_to_float(lohi[2 * t + 1]);
    const float span = hi - lo;
    float f = span > 0.0f ? (x[i * d + t] - lo) / span * levels : 0.0f;
    f = fminf(fmaxf(f, 0.0f), levels - 1.0f);
    q[t] = static_cast<uint32_t>(f);
  }
  uint32_t k = 0;
  for (int b = bits - 1; b >= 0; --b)
    for (int t = 0; t < m; ++t) k = (k << 1) | ((q[t] >> b) & 1u);
  key[i] = k;
  val[i] = static_cast<int32_t>(i);
}

// Batch-major variant: key = (row batch of the original index) << 32 | Morton code, so the points
// of row batch b occupy exactly positions [b * batch_rows, (b + 1) * batch_rows) of the order,
// Z-ordered among themselves (the memory-bounded fit evaluates one batch's tile range at a time).
__global__ void batch_key_kernel(const uint32_t* __restrict__ morton, int64_t n, int64_t batch_rows,
                                 unsigned long long* __restrict__ key)
{
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  key[i] = (static_cast<unsigned long long>(i / batch_rows) << 32) | morton[i];
}

size_t order_scratch_bytes(int64_t n)
{
  size_t temp32 = 0, temp64 = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, temp32, static_cast<const uint32_t*>(nullptr),
                                  static_cast<uint32_t*>(nullptr), static_cast<const int32_t*>(nullptr),
                                  static_cast<int32_t*>(nullptr), static_cast<int>(n));
  cub::DeviceRadixSort::SortPairs(nullptr, temp64, static_cast<const unsigned long long*>(nullptr),
                                  static_cast<unsigned long long*>(nullptr), static_cast<const int32_t*>(nullptr),
                                  static_cast<int32_t*>(nullptr), static_cast<int>(n));
  // 32-bit keys in/out + values in + two 64-bit key arrays (batch-major order) + the sort's
  // temporary storage + the bounding box
  return align_up(sizeof(uint32_t) * n, 256) * 3 + align_up(sizeof(unsigned long long) * n, 256) * 2 +
         align_up(std::max(temp32, temp64), 256) + 256;
}

// perm[r] = original index of the r-th point in Z-order of the leading coordinates; with
// batch_rows > 0, batch-major: row batch first (original index / batch_rows), then Z-order.
Status spatial_order(const float* x, int64_t n, int32_t d, int32_t* perm, void* scratch, size_t scratch_bytes,
                     cudaStream_t s, int64_t batch_rows)
{
  if (scratch_bytes < order_scratch_bytes(n)) return Status::Err(DBM_ERR_INVALID, "order scratch too small");
  const int m = d < 4 ? d : 4;
  unsigned char* p = static_cast<unsigned char*>(scratch);
  const size_t kb = align_up(sizeof(uint32_t) * n, 256);
  const size_t kb64 = align_up(sizeof(unsigned long long) * n, 256);
  uint32_t* keys_in = reinterpret_cast<uint32_t*>(p);
  uint32_t* keys_out = reinterpret_cast<uint32_t*>(p + kb);
  int32_t* vals_in = reinterpret_cast<int32_t*>(p + 2 * kb);
  unsigned long long* bkeys_in = reinterpret_cast<unsigned long long*>(p + 3 * kb);
  unsigned long long* bkeys_out = reinterpret_cast<unsigned long long*>(p + 3 * kb + kb64);
  uint32_t* lohi = reinterpret_cast<uint32_t*>(p + 3 * kb + 2 * kb64);
  void* temp = p + 3 * kb + 2 * kb64 + 256;
  size_t temp_bytes = scratch_bytes - 3 * kb - 2 * kb64 - 256;
  count_launch(3);
  bbox_init_kernel<<<1, 32, 0, s>>>(lohi);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(ceil_div(n, 256), 1184));
  bbox_kernel<<<blocks, 256, 0, s>>>(x, n, d, m, lohi);
  morton_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(x, n, d, m, lohi, keys_in, vals_in);
  DBM_CUDA(cudaGetLastError());
  if (batch_rows > 0) {
    count_launch();
    batch_key_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, s>>>(keys_in, n, batch_rows, bkeys_in);
    DBM_CUDA(cudaGetLastError());
    int end_bit = 33;  // batch ids below 2^(end_bit - 32)
    while ((int64_t(1) << (end_bit - 32)) <= ceil_div(n, batch_rows)) ++end_bit;
    DBM_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, bkeys_in, bkeys_out, vals_in, perm,
                                             static_cast<int>(n), 0, end_bit, s));
    return Status::Ok();
  }
  DBM_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, vals_in, perm,
                                           static_cast<int>(n), 0, 32, s));
  return Status::Ok();
}

}  // namespace dbm
