// prune.cu -- exact tile-pair pruning for the distance pass.
//
// For every 128-point tile I of the (Z-ordered) points, lo[I][t] / hi[I][t] bound its points'
// coordinates in each dim t.  For a tile pair (I, J) and any a in tile I, b in tile J:
//   |fl(a_t - b_t)| >= g_t = max(0, fl(lo_J[t] - hi_I[t]), fl(lo_I[t] - hi_J[t]))
// because round-to-nearest is monotone and symmetric.  The distance kernel accumulates
// acc = fma(d_t, d_t, acc) over t = 0..D-1, which is monotone in |d_t| and in acc, so the same
// chain over the gaps, lb = fma(g_t, g_t, lb), is a lower bound of every pair's computed acc
// at every prefix.  Once lb > eps2[k-1] no pair of the tile pair can be a neighbour under any
// eps: the tile pair is skipped without evaluating a single pair, and nothing else changes.
//
// Surviving tile pairs go to a worklist in tile-pair order (two passes: per-block counts,
// scan, ordered write), so every rank of a sharded run sees the same list and takes an equal
// slice of it.  Entries are the tile coordinates packed as J << 32 | I.
#include "dbm_internal.cuh"

#include <algorithm>

namespace dbm {

constexpr int kPruneThreads = 256;
constexpr int kPruneItems = 16;  // tile pairs per thread per block pass
constexpr int64_t kPruneBlock = static_cast<int64_t>(kPruneThreads) * kPruneItems;

// One warp per (tile, dim): min / max over the tile's valid points (columns < n of XT).
__global__ void tile_box_kernel(const float* __restrict__ xt, int64_t n, int64_t npad, int32_t d,
                                int64_t tiles, float* __restrict__ lo, float* __restrict__ hi)
{
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= tiles * d) return;
  const int64_t tile = w / d;
  const int32_t t = static_cast<int32_t>(w - tile * d);
  float mn = INFINITY, mx = -INFINITY;
  for (int r = lane; r < 128; r += 32) {
    const int64_t i = tile * 128 + r;
    if (i < n) {
      const float v = xt[static_cast<int64_t>(t) * npad + i];
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  if (lane == 0) {
    lo[tile * d + t] = mn;
    hi[tile * d + t] = mx;
  }
}

__device__ __forceinline__ void prune_tri_coords(long long c, long long& I, long long& J)
{
  long long j = static_cast<long long>((sqrt(8.0 * static_cast<double>(c) + 1.0) - 1.0) * 0.5);
  while (j * (j + 1) / 2 > c) --j;
  while ((j + 1) * (j + 2) / 2 <= c) ++j;
  J = j;
  I = c - j * (j + 1) / 2;
}

// true when some pair of the tile pair may be within cutoff
__device__ __forceinline__ bool tile_pair_survives(long long I, long long J, const float* __restrict__ lo,
                                                   const float* __restrict__ hi, int32_t d, float cutoff)
{
  if (I == J) return true;
  const float* loI = lo + I * d;
  const float* hiI = hi + I * d;
  const float* loJ = lo + J * d;
  const float* hiJ = hi + J * d;
  float lb = 0.0f;
  for (int32_t t = 0; t < d; ++t) {
    const float g = fmaxf(0.0f, fmaxf(__fsub_rn(loJ[t], hiI[t]), __fsub_rn(loI[t], hiJ[t])));
    lb = __fmaf_rn(g, g, lb);
    if (lb > cutoff) return false;
  }
  return true;
}

template <bool WRITE>
__global__ void tile_prune_kernel(int64_t pairs, const float* __restrict__ lo, const float* __restrict__ hi,
                                  int32_t d, float cutoff, int32_t* __restrict__ block_counts,
                                  const int64_t* __restrict__ block_offsets, long long* __restrict__ work)
{
  __shared__ int32_t warp_tot[kPruneThreads / 32];
  const int64_t b0 = static_cast<int64_t>(blockIdx.x) * kPruneBlock;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t base = WRITE ? block_offsets[blockIdx.x] : 0;
  int32_t total = 0;
  // items are taken in tile-pair order: round q covers [b0 + q*256, b0 + (q+1)*256)
  for (int q = 0; q < kPruneItems; ++q) {
    const long long c = b0 + static_cast<int64_t>(q) * kPruneThreads + threadIdx.x;
    long long I = 0, J = 0;
    if (c < pairs) prune_tri_coords(c, I, J);
    const bool keep = c < pairs && tile_pair_survives(I, J, lo, hi, d, cutoff);
    const uint32_t bal = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int32_t before = 0, round = 0;
    for (int w2 = 0; w2 < kPruneThreads / 32; ++w2) {
      if (w2 < warp) before += warp_tot[w2];
      round += warp_tot[w2];
    }
    if (WRITE && keep) work[base + total + before + __popc(bal & ((1u << lane) - 1u))] = (J << 32) | I;
    total += round;
    __syncthreads();
  }
  if (!WRITE && threadIdx.x == 0) block_counts[blockIdx.x] = total;
}

int64_t prune_blocks(int64_t pairs) { return ceil_div(pairs, kPruneBlock); }

Status launch_tile_boxes(const float* xt, int64_t n, int64_t npad, int32_t d, float* lo, float* hi, cudaStream_t s)
{
  const int64_t tiles = ceil_div(n, 128);
  const int64_t warps = tiles * d;
  count_launch();
  tile_box_kernel<<<static_cast<unsigned>(ceil_div(warps * 32, 256)), 256, 0, s>>>(xt, n, npad, d, tiles, lo, hi);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// pass 1: per-block survivor counts and their exclusive scan (offsets[nb] = total)
Status launch_prune_count(int64_t pairs, const float* lo, const float* hi, int32_t d, float cutoff,
                          int32_t* counts, int64_t* offsets, void* scan_scratch, size_t scan_bytes,
                          cudaStream_t s)
{
  const int64_t nb = prune_blocks(pairs);
  count_launch();
  tile_prune_kernel<false><<<static_cast<unsigned>(nb), kPruneThreads, 0, s>>>(pairs, lo, hi, d, cutoff, counts,
                                                                                nullptr, nullptr);
  DBM_CUDA(cudaGetLastError());
  return exclusive_scan_i32(counts, offsets, nb, scan_scratch, scan_bytes, s);
}

// pass 2: surviving tile-pair indices, in tile-pair order
Status launch_prune_write(int64_t pairs, const float* lo, const float* hi, int32_t d, float cutoff,
                          const int64_t* offsets, long long* work, cudaStream_t s)
{
  const int64_t nb = prune_blocks(pairs);
  count_launch();
  tile_prune_kernel<true><<<static_cast<unsigned>(nb), kPruneThreads, 0, s>>>(pairs, lo, hi, d, cutoff, nullptr,
                                                                              offsets, work);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

}  // namespace dbm
