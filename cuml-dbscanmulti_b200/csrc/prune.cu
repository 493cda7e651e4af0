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
// Surviving tile pairs form a worklist ordered by J, then I (one bound pass writing per-unit keep
// masks and counts, a scan, an ordered expansion of the masks), so every rank of a sharded run sees the same list and takes an equal slice
// of it.  Entries are the tile coordinates packed as J << 32 | I.  Boxes are stored dim-major
// (lo[t * tiles + I]) so that the 32 lanes of a warp, testing 32 consecutive tiles I against
// one J, read consecutive addresses.
#include "dbm_internal.cuh"

#include <algorithm>

namespace dbm {

// One warp per (tile, dim): min / max over the tile's valid points (columns < n of XT),
// written dim-major: lo[t * tiles + tile].
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
    lo[static_cast<int64_t>(t) * tiles + tile] = mn;
    hi[static_cast<int64_t>(t) * tiles + tile] = mx;
  }
}

// Work units: (J, block of kUnitTiles consecutive tiles I <= J), J-major, blocks ascending, so
// that the units' outputs concatenated in unit order are the worklist (J, then I ascending).
constexpr int64_t kUnitTiles = 128;

// units before tile J: sum over j < J of (j / kUnitTiles + 1), in closed form
__host__ __device__ __forceinline__ int64_t units_before(int64_t J)
{
  const int64_t q = J / kUnitTiles, r = J % kUnitTiles;
  return J + kUnitTiles * q * (q - 1) / 2 + q * r;
}

__device__ __forceinline__ void unit_coords(int64_t u, int64_t tiles, int64_t& J, int64_t& blk)
{
  // tile J = K q + r (K = kUnitTiles) owns q + 1 units, and the units before J = K q number
  // K q (q + 1) / 2: q from the square root (corrected by +-1 for rounding), then r and blk by
  // division
  (void)tiles;
  constexpr int64_t K = kUnitTiles;
  int64_t q = static_cast<int64_t>((sqrt(1.0 + 8.0 * static_cast<double>(u) / K) - 1.0) * 0.5);
  while (q > 0 && K * q * (q + 1) / 2 > u) --q;
  while (K * (q + 1) * (q + 2) / 2 <= u) ++q;
  const int64_t rem = u - K * q * (q + 1) / 2;
  J = kUnitTiles * q + rem / (q + 1);
  blk = rem % (q + 1);
}

// One warp per unit: the tiles I of the unit's block (I <= J) whose boxes may meet J's (I == J
// always).  The bound's chain runs over the dims in order and is checked after each group of
// dims loaded together (lb only grows along the dims, so stopping later is as exact).  The
// first 4 dims of all four 32-tile steps are loaded and chained together (one round of L2
// latency per unit: the Z-order sorts these dims, so they drop most tile pairs), then each step
// with survivors continues its chains from dim 4, 8 dims per round of loads.  Writes the unit's
// keep mask (bit q of word c: I = block start + 32 c + q) and its count.
__global__ void tile_pairs_kernel(int64_t tiles, int64_t u0, int64_t u1, const float* __restrict__ lo,
                                  const float* __restrict__ hi, int32_t d, float cutoff, int32_t* __restrict__ counts,
                                  uint32_t* __restrict__ masks)
{
  constexpr int kSteps = static_cast<int>(kUnitTiles / 32);
  const int64_t u = u0 + ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (u >= u1) return;
  int64_t J, blk;
  unit_coords(u, tiles, J, blk);
  int32_t total = 0;
  const int64_t i0 = blk * kUnitTiles;
  const int64_t i1 = i0 + kUnitTiles - 1 < J ? i0 + kUnitTiles - 1 : J;
  float jl[4], jh[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    jl[q] = q < d ? __ldg(lo + static_cast<int64_t>(q) * tiles + J) : 0.0f;
    jh[q] = q < d ? __ldg(hi + static_cast<int64_t>(q) * tiles + J) : 0.0f;
  }
  float lb0[kSteps];
  bool live[kSteps];
#pragma unroll
  for (int c = 0; c < kSteps; ++c) {
    const int64_t I = i0 + 32 * c + lane;
    live[c] = I <= i1 && I != J;
    float gq[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      gq[q] = 0.0f;
      if (live[c] && q < d) {
        const int64_t ti = static_cast<int64_t>(q) * tiles;
        gq[q] = fmaxf(0.0f, fmaxf(__fsub_rn(jl[q], __ldg(hi + ti + I)), __fsub_rn(__ldg(lo + ti + I), jh[q])));
      }
    }
    float lb = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) lb = __fmaf_rn(gq[q], gq[q], lb);
    lb0[c] = lb;
  }
#pragma unroll
  for (int c = 0; c < kSteps; ++c) {
    const int64_t I = i0 + 32 * c + lane;
    bool keep = I <= i1;
    if (live[c]) {
      float lb = lb0[c];
      if (lb > cutoff) keep = false;
      for (int32_t t0 = 4; keep && t0 < d; t0 += 8) {
        float gq[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int32_t t = t0 + q;
          gq[q] = 0.0f;
          if (t < d) {
            const int64_t ti = static_cast<int64_t>(t) * tiles;
            gq[q] = fmaxf(0.0f, fmaxf(__fsub_rn(__ldg(lo + ti + J), __ldg(hi + ti + I)),
                                      __fsub_rn(__ldg(lo + ti + I), __ldg(hi + ti + J))));
          }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) lb = __fmaf_rn(gq[q], gq[q], lb);
        if (lb > cutoff) {
          keep = false;
          break;
        }
      }
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) masks[u * (kUnitTiles / 32) + c] = bal;
    total += __popc(bal);
  }
  if (lane == 0) counts[u] = total;
}

// One warp per unit: its kept tiles as packed worklist entries at off[u] ..., I ascending.
__global__ void tile_pairs_write_kernel(int64_t tiles, int64_t units, const uint32_t* __restrict__ masks,
                                        const int64_t* __restrict__ off, long long* __restrict__ work, int64_t cap)
{
  const int64_t u = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (u >= units) return;
  int64_t J, blk;
  unit_coords(u, tiles, J, blk);
  int64_t at = off[u];
#pragma unroll
  for (int c = 0; c < static_cast<int>(kUnitTiles / 32); ++c) {
    const uint32_t m = masks[u * (kUnitTiles / 32) + c];
    const int64_t idx = at + __popc(m & ((1u << lane) - 1u));
    if (((m >> lane) & 1u) && idx < cap) work[idx] = (J << 32) | (blk * kUnitTiles + 32 * c + lane);
    at += __popc(m);
  }
}

// ---- host side ----------------------------------------------------------------------------------

int64_t prune_units(int64_t tiles) { return units_before(tiles); }

size_t prune_scratch_bytes(int64_t tiles, int32_t d)
{
  (void)d;
  const int64_t units = units_before(tiles);
  return align_up(sizeof(int32_t) * units, 256) + align_up(sizeof(int64_t) * (units + 1), 256) +
         align_up(sizeof(uint32_t) * units * (kUnitTiles / 32), 256);
}

Status launch_tile_boxes(const float* xt, int64_t n, int64_t npad, int32_t d, float* lo, float* hi, cudaStream_t s)
{
  const int64_t tiles = ceil_div(n, 128);
  const int64_t warps = tiles * d;
  count_launch();
  tile_box_kernel<<<static_cast<unsigned>(ceil_div(warps * 32, 256)), 256, 0, s>>>(xt, n, npad, d, tiles, lo, hi);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// The bound pass over the units [u0, u1) only: their keep masks (kUnitTiles / 32 words per unit)
// and counts, at their unit positions of the full-size arrays (a multi-GPU rank bounds its share
// and the ranks all-gather the rest).
Status launch_prune_bound(int64_t tiles, const float* lo, const float* hi, int32_t d, float cutoff, int64_t u0,
                          int64_t u1, int32_t* counts, uint32_t* masks, cudaStream_t s)
{
  if (u1 <= u0) return Status::Ok();
  count_launch();
  tile_pairs_kernel<<<static_cast<unsigned>(ceil_div((u1 - u0) * 32, 256)), 256, 0, s>>>(tiles, u0, u1, lo, hi, d,
                                                                                       cutoff, counts, masks);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// Per-unit counts and their scan: afterwards the worklist length is at *count_out_dev.  With
// ext_counts / ext_masks (all units, e.g. gathered from every rank), the bound pass is skipped.
Status launch_prune_count(int64_t tiles, const float* lo, const float* hi, int32_t d, float cutoff, void* scratch,
                          size_t scratch_bytes, void* scan_scratch, size_t scan_bytes, const int64_t** count_out_dev,
                          cudaStream_t s, const int32_t* ext_counts)
{
  if (scratch_bytes < prune_scratch_bytes(tiles, d)) return Status::Err(DBM_ERR_INVALID, "prune scratch too small");
  const int64_t units = units_before(tiles);
  unsigned char* sp = static_cast<unsigned char*>(scratch);
  int32_t* counts = reinterpret_cast<int32_t*>(sp);
  int64_t* off = reinterpret_cast<int64_t*>(sp + align_up(sizeof(int32_t) * units, 256));
  uint32_t* masks = reinterpret_cast<uint32_t*>(sp + align_up(sizeof(int32_t) * units, 256) +
                                                align_up(sizeof(int64_t) * (units + 1), 256));
  if (!ext_counts) DBM_TRY(launch_prune_bound(tiles, lo, hi, d, cutoff, 0, units, counts, masks, s));
  DBM_TRY(exclusive_scan_i32(ext_counts ? ext_counts : counts, off, units, scan_scratch, scan_bytes, s));
  *count_out_dev = off + units;
  return Status::Ok();
}

// the packed worklist entries, J ascending then I ascending (the first `cap` of them), from the
// scratch's masks or ext_masks
Status launch_prune_write(int64_t tiles, const float* lo, const float* hi, int32_t d, float cutoff, void* scratch,
                          long long* work, int64_t cap, cudaStream_t s, const uint32_t* ext_masks)
{
  (void)lo;
  (void)hi;
  (void)d;
  (void)cutoff;
  const int64_t units = units_before(tiles);
  const unsigned char* sp = static_cast<const unsigned char*>(scratch);
  const int64_t* off = reinterpret_cast<const int64_t*>(sp + align_up(sizeof(int32_t) * units, 256));
  const uint32_t* masks = ext_masks ? ext_masks
                                    : reinterpret_cast<const uint32_t*>(sp + align_up(sizeof(int32_t) * units, 256) +
                                                                        align_up(sizeof(int64_t) * (units + 1), 256));
  count_launch();
  tile_pairs_write_kernel<<<static_cast<unsigned>(ceil_div(units * 32, 256)), 256, 0, s>>>(tiles, units, masks, off,
                                                                                         work, cap);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

int64_t prune_mask_words() { return kUnitTiles / 32; }

}  // namespace dbm
