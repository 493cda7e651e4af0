// dist_tc.cu -- screened distance pass: a tensor-core bound picks the candidate pairs of a tile
// pair, the exact fp32 chain decides every one of them.
//
// The reference's per-pair arithmetic (src/multi/eps_neighborhood.cuh:151-168: acc =
// fma(q[t]-p[t], q[t]-p[t], acc) in dim order, code = smallest e with acc <= eps2[e]) costs
// 2*D CUDA-core operations per pair.  In the sparse regime almost every pair of a surviving
// tile pair is far beyond the largest eps, so this kernel first bounds all 128 x 128 pairs with
// one tf32 tcgen05 GEMM and evaluates the exact chain only for the pairs the bound cannot
// exclude.  Nothing about the results changes: a pair is a neighbour iff its exact chain says
// so, and the bound provably never drops a neighbour (argument below).
//
// Bound.  For the tile pair (I, J) let c be tile J's box centre and, for each point p of both
// tiles, a_p = tf32(fl(x_p - c)) (per coordinate, round to nearest; |a_p - (x_p - c)| <= rho |a_p|
// with rho = 0.00049 covering the fp32 subtraction and the 11-bit tf32 rounding).  With
// E = eps2[k-1]:
//   acc(i,j) <= E  =>  |x_i - x_j| <= s := sqrt(E (1 + (D+3) 2^-24))   (the fma chain is
//                      monotone and each step loses at most a factor (1 - 2^-24))
//                  =>  |a_i - a_j| <= s + rho (r_i + r_j),   r_p >= |a_p| (per row)
//                  =>  |a_i - a_j|^2 <= s^2 + (2 s rho r_i + 2 rho^2 r_i^2) + (2 s rho r_j + 2 rho^2 r_j^2)
// using (u + v)^2 <= 2u^2 + 2v^2 for the perturbation.  With |a_i - a_j|^2 = n_i + m_j - 2 a_i.a_j
// (n_i = |a_i|^2, m_j = |a_j|^2, computed in fp32) a neighbour has
//   V_ij = a_i.a_j - h_i - g_j > 0,
//   h_i = (n_i - s^2 - 2 s rho r_i - 2 rho^2 r_i^2) / 2 - 2^-13 (n_i + s^2),
//   g_j = (m_j - 2 s rho r_j - 2 rho^2 r_j^2) / 2 - 2^-13 m_j,
// where the 2^-13 margins exceed 5x every rounding error of n_i, m_j, h_i, g_j and of the
// tensor core's fp32 accumulation over K <= 72 products (at most K 2^-22 of the sum of the
// magnitudes of the terms, which is <= n_i + m_j + s^2).  Each row's slack depends only on its
// own norm, so a far-away point loosens nothing but its own pairs.  The GEMM computes V
// directly: the K dimension carries the D centred coordinates, then -h_i split into two tf32
// terms against ones, then ones against -g_j split the same way.  A pair is a candidate iff the
// fp32 result has a clear sign bit; 32 results are tested at once by AND-ing their bit patterns.
//
// Per CTA (128 threads; thread r owns row r of tile I and column r of tile J), persistent over
// the worklist:
//   rows:   one TMA load stages tile I's fp32 rows ({128 points, KP dims} of XT) in the
//           operand-A buffer, issued as soon as the previous MMA has read that buffer; thread r
//           copies its row to registers, and after a barrier the operand is built in place;
//   build:  centred tf32 operands in the canonical K-major no-swizzle layout (8-row x 16-byte
//           core matrices; LBO = 2048 B between the two K halves of an MMA, SBO = 128 B
//           between 8-row groups) plus the h / g columns; tile J (operand, and for D <= 36 an
//           fp32 copy in shared memory) only when J changes;
//   MMA:    KS x tcgen05.mma.cta_group::1.kind::tf32 (M = N = 128, K = 8) into 128 TMEM
//           columns, committed to an mbarrier;
//   screen: tcgen05.ld 32x32b.x64 (x32 for D <= 20) -> per-thread candidate masks;
//   exact:  thread r runs the fp32 chain for each of its candidates from its registers and the
//           fp32 tile J (shared memory, or XT for D > 36), then code, COO word and per-code
//           histogram (dist_tri_kernel's outputs).
// A tile pair whose bound admits more than kScreenCap candidates (kScreenCapXT above D = 36;
// dense regime), or whose coordinates are too large for the bound, is appended to a fallback
// list for dist_tri_kernel.
#include "dbm_internal.cuh"

#include <algorithm>
#include <cmath>

namespace dbm {

constexpr int kScreenTile = 128;
constexpr int kScreenThreads = 128;
constexpr int kScreenCap = 1024;        // candidates per tile pair before the fallback
// ... above D = 36, where each candidate's exact chain reads tile J's row from L2: a tile pair
// with that many candidates is cheaper in the exact tile kernel
constexpr int kScreenCapXT = 256;
constexpr int kScreenGrab = 16;         // worklist entries per chunk (one atomic each), at least
constexpr int kScreenGrabMax = 64;      // ... and at most: larger chunks change tile J less often
constexpr uint32_t kScreenPolls = 1u << 24;
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kKHalfBytes = 2048;  // one 4-column (16-byte) K slice of a 128-row operand
constexpr uint32_t kKStepBytes = 2 * kKHalfBytes;  // one MMA: K = 8 tf32 columns
constexpr size_t kScreenMinSmem = 48 * 1024;  // at most 4 CTAs (512 TMEM columns) per SM
constexpr float kRho = 0.00049f;

// instruction descriptor: D f32, A and B tf32, both K-major, M = 128, N = 128
constexpr uint32_t kIdescTf32 = (1u << 4) | (2u << 7) | (2u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

struct ScreenParams {
  int64_t n;
  int64_t npad;
  int32_t d;
  int32_t k;
  int64_t item_count;            // this shard's items (shard_item maps them into the worklist)
  const int64_t* total_dev;      // when set: worklist length on the device (capped at cap),
  int64_t cap;                   // and this shard's slice is computed here
  int32_t shard, nshards;
  const long long* work;
  const float* xt;               // dp x npad, dim-major
  unsigned long long* counters;  // [0] edge cursor, [4] item cursor, [5] fallback count,
                                 // [6] candidates, [7] screened tile pairs
  uint64_t* edges;
  uint64_t edge_cap;
  int32_t* hist;
  int32_t* err;
  const int32_t* perm;
  const float* box_lo;  // d x tiles (dim-major)
  const float* box_hi;
  int64_t tiles;
  long long* fallback;
  int64_t keep_lo, keep_hi;  // emit only pairs with an endpoint at an XT position in [keep_lo, keep_hi)
  float sqrt_e;         // s of the bound, rounded up
  float eps2[kMaxEps];
};

// ---- tcgen05 / TMEM wrappers ------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols)
{
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols)
{
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint64_t smem_desc_kmajor(uint32_t addr)
{
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((kKHalfBytes >> 4) & 0x3FFFu) << 16) |  // LBO: next K half
         (static_cast<uint64_t>((128u >> 4) & 0x3FFFu) << 32) |          // SBO: next 8 rows
         (1ull << 46);                                                   // descriptor version
}
__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate)
{
  asm volatile(
    "{\n\t.reg .pred p;\n\t"
    "setp.ne.b32 p, %3, 0;\n\t"
    "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %4, p;\n\t}" ::"r"(tmem_d),
    "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(kIdescTf32)
    : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane, waited for in the same asm
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[32])
{
  asm volatile(
    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
    "tcgen05.wait::ld.sync.aligned;"
    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
    : "r"(taddr)
    : "memory");
}
// 64 consecutive fp32 columns of this thread's TMEM lane, waited for in the same asm
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[64])
{
  asm volatile(
    "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
    "tcgen05.wait::ld.sync.aligned;"
    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
    : "r"(taddr)
    : "memory");
}

// round to the nearest tf32 value, ties away from zero (the magnitude bits round half up)
__device__ __forceinline__ float tf32_rn(float v)
{
  return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

// worklist entries are J << 32 | I
__device__ __forceinline__ void screen_coords(long long e, long long& I, long long& J)
{
  I = e & 0xffffffffLL;
  J = e >> 32;
}

// ---- operand construction ---------------------------------------------------------------------
// Row r of a 128-row K-major tf32 operand: column t lives at (t / 4) * 2048 + r * 16 + (t % 4) * 4.
// XT holds KP zero-padded rows here, so rows t >= d read as 0.
template <int KP>
__device__ __forceinline__ void load_row(const float* __restrict__ xt, int64_t npad, int64_t col, bool valid,
                                         float (&v)[KP])
{
  const float* q = xt + col;
#pragma unroll
  for (int t = 0; t < KP; ++t) {
    v[t] = valid ? __ldg(q) : 0.0f;
    q += npad;
  }
}

// Writes the centred tf32 coordinates (zeros past d: x and the centre are 0 there) and returns
// the fp32 sum of their squares.  The centre comes in registers: read from shared memory inside
// this loop, each load would wait behind the preceding operand stores (they may alias).
template <int KP>
__device__ __forceinline__ float build_row(const float (&x)[KP], const float (&cs)[KP], int r, unsigned char* op)
{
  float nq[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four partial sums: independent FMA chains
#pragma unroll
  for (int ch = 0; ch < KP / 4; ++ch) {
    float w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int t = ch * 4 + h;
      w[h] = tf32_rn(__fsub_rn(x[t], cs[t]));
      nq[h] = __fmaf_rn(w[h], w[h], nq[h]);
    }
    *reinterpret_cast<float4*>(op + ch * kKHalfBytes + r * 16) = make_float4(w[0], w[1], w[2], w[3]);
  }
  return __fadd_rn(__fadd_rn(nq[0], nq[1]), __fadd_rn(nq[2], nq[3]));
}

__device__ __forceinline__ void put_f32(unsigned char* op, int r, int t, float v)
{
  *reinterpret_cast<float*>(op + (t >> 2) * kKHalfBytes + r * 16 + (t & 3) * 4) = v;
}

// columns d, d+1 = split(-h) (A side) or ones (B side); d+2, d+3 = ones (A) or split(-g) (B);
// v ~ t1 + t2 to about 2^-22 |v| (the residual is exact in fp32)
__device__ __forceinline__ void put_ext(unsigned char* op, int r, int d, bool a_side, float v)
{
  const float t1 = tf32_rn(-v);
  const float t2 = tf32_rn(__fsub_rn(-v, t1));
  const int s0 = a_side ? d : d + 2;
  const int s1 = a_side ? d + 2 : d;
  put_f32(op, r, s0, t1);
  put_f32(op, r, s0 + 1, t2);
  put_f32(op, r, s1, 1.0f);
  put_f32(op, r, s1 + 1, 1.0f);
}

// h_i and g_j of the bound for a row / column with squared norm n (r = sqrt(n (1 + 2^-16))
// rounded up bounds the exact norm, which the fp32 sum of squares can underestimate by <= 2^-17)
__device__ __forceinline__ float norm_slack(float n, float se)
{
  const float r = __fsqrt_ru(__fmul_ru(n, 1.0000153f));
  return __fmul_ru(__fmul_ru(2.0f * kRho, r), __fadd_ru(se, __fmul_ru(kRho, r)));  // 2 s rho r + 2 rho^2 r^2
}
__device__ __forceinline__ float row_slack(float n, float se)
{
  const float s2 = __fmul_ru(se, se);
  const float h = 0.5f * __fsub_rd(__fsub_rd(n, s2), norm_slack(n, se));
  return __fsub_rd(h, __fmul_ru(0.0001220703125f, __fadd_ru(n, s2)));
}
__device__ __forceinline__ float col_slack(float m, float se)
{
  const float g = 0.5f * __fsub_rd(m, norm_slack(m, se));
  return __fsub_rd(g, __fmul_ru(0.0001220703125f, m));
}

// build_row for a row read straight from XT four dims at a time; an invalid row is centred to 0
template <int KP>
__device__ __forceinline__ float build_row_xt(const float* __restrict__ xt, int64_t npad, int64_t col, bool valid,
                                              const float* __restrict__ cs, int r, unsigned char* op)
{
  float nq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const float* q = xt + col;
#pragma unroll
  for (int ch = 0; ch < KP / 4; ++ch) {
    float w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int t = ch * 4 + h;
      const float x = valid ? __ldg(q + t * npad) : cs[t];
      w[h] = tf32_rn(__fsub_rn(x, cs[t]));
      nq[h] = __fmaf_rn(w[h], w[h], nq[h]);
    }
    *reinterpret_cast<float4*>(op + ch * kKHalfBytes + r * 16) = make_float4(w[0], w[1], w[2], w[3]);
  }
  return __fadd_rn(__fadd_rn(nq[0], nq[1]), __fadd_rn(nq[2], nq[3]));
}

template <int KS>
__global__ void __launch_bounds__(kScreenThreads, (KS <= 3 ? 4 : (KS <= 5 ? 3 : 2)))
dist_screen_kernel(const __grid_constant__ CUtensorMap xt_map, const ScreenParams p)
{
  constexpr int KP = 8 * KS;
  // Up to D = 36 tile J's fp32 rows stay in shared memory for the exact chain; above that they
  // are read from XT (L2) instead, which halves the CTA's shared memory and fits two CTAs per SM.
  constexpr bool kSmemJ = KS <= 5;
  // wider TMEM loads wait less often; the narrow ones keep small-D instances at 4 CTAs per SM
  constexpr int kLdCols = KS <= 3 ? 32 : 64;
  constexpr uint32_t kStageBytes = KP * kScreenTile * sizeof(float);  // == KS * kKStepBytes
  extern __shared__ unsigned char dyn_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dyn_raw) + 1023) & ~uintptr_t(1023));
  // Tile I arrives by TMA as fp32 [KP][128] in the operand-A buffer; every thread copies its row
  // to registers and, after a barrier, writes the operand over it in place.
  unsigned char* opA = base;
  const float* stage = reinterpret_cast<const float*>(opA);
  unsigned char* opB = opA + KS * kKStepBytes;
  float* xJ = reinterpret_cast<float*>(opB + KS * kKStepBytes);  // [KP][128] fp32 of tile J
  uint32_t* hitq = reinterpret_cast<uint32_t*>(xJ + (kSmemJ ? KP * kScreenTile : 0));  // [2][kScreenCap]

  __shared__ __align__(8) uint64_t bar_mma;
  __shared__ __align__(8) uint64_t bar_tma;
  __shared__ uint32_t s_tmem;
  __shared__ long long s_chunk[2];  // worklist start of the current / next chunk of this CTA
  __shared__ int s_clen[2];         // ... and its length
  __shared__ int s_cnt[2], s_hits[2];
  __shared__ int s_badJ;
  __shared__ float s_c[72];
  __shared__ float s_eps2[kMaxEps];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int d = p.d;
  const int64_t n = p.n;
  const float cutoff = p.eps2[p.k - 1];
  const float se = p.sqrt_e;
  int64_t item_count = p.item_count;
  if (p.total_dev) {
    const int64_t total = *p.total_dev < p.cap ? *p.total_dev : p.cap;
    item_count = shard_items(total, p.shard, p.nshards);
  }
  if (tid < kMaxEps) s_eps2[tid] = p.eps2[tid];
  if (warp == 0) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_tma, 1);
    mbar_fence_init();
    s_cnt[0] = s_cnt[1] = 0;
    s_hits[0] = s_hits[1] = 0;
    s_badJ = 0;
  }
  // Chunks shrink with the work left (an eighth of it spread over the grid, clamped to
  // [kScreenGrab, kScreenGrabMax]): long runs of one tile J while there is plenty of work, a short
  // tail.  Thread 0 grabs; `seen` is the cursor as it last saw it.
  // A chunk grabbed at a chunk boundary is needed only near the end of the following chunk, so
  // its cursor value is stored one item later and the atomic's latency stays off the item path.
  long long seen = 0, pend_c = 0;
  int pend_slot = -1, pend_g = 0;
  auto grab = [&](int slot) {
    long long g = (item_count - seen) / (8LL * gridDim.x);
    g = g < kScreenGrab ? kScreenGrab : (g > kScreenGrabMax ? kScreenGrabMax : g);
    pend_c = static_cast<long long>(atomicAdd(p.counters + 4, static_cast<unsigned long long>(g)));
    pend_g = static_cast<int>(g);
    pend_slot = slot;
  };
  auto publish = [&]() {
    if (pend_slot >= 0) {
      s_chunk[pend_slot] = pend_c;
      s_clen[pend_slot] = pend_g;
      seen = pend_c + pend_g;
      pend_slot = -1;
    }
  };
  if (tid == 0) {
    grab(0);
    publish();
    grab(1);
    publish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);

  // The CTA's items: chunks of consecutive worklist entries, each chunk grabbed one ahead.
  long long cstart = s_chunk[0];
  int clen = s_clen[0];
  int pos = 0, m = 0;
  auto item_index = [&](int q) -> long long {  // q-th item from the current chunk's start (q <= clen + 1)
    return q < clen ? cstart + q : s_chunk[(m + 1) & 1] + (q - clen);
  };
  auto load_entry = [&](long long idx) -> long long {
    return idx < item_count ? __ldg(p.work + shard_item(idx, p.shard, p.nshards)) : -1;
  };
  long long e_cur = load_entry(item_index(0));
  long long e_nxt = e_cur >= 0 ? load_entry(item_index(1)) : -1;

  uint32_t ph_mma = 0, ph_tma = 0;
  bool tma_pending = false;  // a stage load is in flight (tracked by thread 0)
  if (tid == 0 && e_cur >= 0) {
    mbar_arrive_expect_tx(&bar_tma, kStageBytes);
    tma_load_2d(opA, &xt_map, static_cast<int32_t>((e_cur & 0xffffffffLL) * kScreenTile), 0, &bar_tma);
    tma_pending = true;
  }
  long long curJ = -1;
  unsigned long long my_candidates = 0, my_screened = 0;
  bool failed = false;
  int par = 0;
  // Neighbour pairs of an item are queued in shared memory (hitq[par]) and written out during the
  // next item's MMA: each warp takes a contiguous quarter of the queue and one edge-cursor atomic.
  int32_t prev_row0 = 0, prev_col0 = 0;
  auto flush = [&](int slot) {
    const int nh = s_hits[slot];
    const int q0 = nh * warp / (kScreenThreads / 32), q1 = nh * (warp + 1) / (kScreenThreads / 32);
    if (q1 <= q0) return;
    unsigned long long b0 = 0;
    if (lane == 0) b0 = atomicAdd(p.counters, static_cast<unsigned long long>(q1 - q0));
    b0 = __shfl_sync(0xffffffffu, b0, 0);
    for (int q = q0 + lane; q < q1; q += 32) {
      const uint32_t e = hitq[slot * kScreenCap + q];
      const int code = static_cast<int>(e >> 28);
      const int32_t oi = p.perm[prev_row0 + static_cast<int>((e >> 8) & 0xffu)];
      const int32_t oj = p.perm[prev_col0 + static_cast<int>(e & 0xffu)];
      const int32_t lo = min(oi, oj), hi = max(oi, oj);
      const unsigned long long idx = b0 + static_cast<unsigned long long>(q - q0);
      if (idx < p.edge_cap)
        p.edges[idx] = (static_cast<uint64_t>(lo) << 32) | (static_cast<uint64_t>(code) << kCodeShift) |
                       static_cast<uint64_t>(hi);
      if (p.hist) {
        int32_t* hrow = p.hist + static_cast<int64_t>(code) * n;
        atomicAdd(hrow + oi, 1);
        atomicAdd(hrow + oj, 1);
      }
    }
  };

  while (e_cur >= 0) {
    const long long e_nn = e_nxt >= 0 ? load_entry(item_index(pos + 2)) : -1;  // two items ahead
    long long I, J;
    screen_coords(e_cur, I, J);
    const bool diag = (I == J);
    const int rows_i = static_cast<int>(n - I * kScreenTile < kScreenTile ? n - I * kScreenTile : kScreenTile);
    const int cols_j = static_cast<int>(n - J * kScreenTile < kScreenTile ? n - J * kScreenTile : kScreenTile);

    // ---- tile I: staged fp32 rows -> registers ----
    const bool staged = mbar_wait_bounded(&bar_tma, ph_tma, kScreenPolls);
    float xr[KP];  // this thread's row of tile I
#pragma unroll
    for (int t = 0; t < KP; ++t) xr[t] = stage[t * kScreenTile + tid];
    // every thread has read the stage (the operand overwrites it), and the previous item's
    // readers of xJ / s_c are done
    if (__syncthreads_or(!staged)) {
      failed = true;
      break;
    }
    ph_tma ^= 1u;
    if (tid == 0) tma_pending = false;

    // ---- tile J (operand B, fp32 copy, centre) when it changes ----
    if (J != curJ) {
      if (tid < KP) s_c[tid] = tid < d ? 0.5f * (p.box_lo[tid * p.tiles + J] + p.box_hi[tid * p.tiles + J]) : 0.0f;
      const bool valid = tid < cols_j;
      float mj;
      if constexpr (kSmemJ) {
        float xj[KP];
        load_row<KP>(p.xt, p.npad, J * kScreenTile + tid, valid, xj);
#pragma unroll
        for (int t = 0; t < KP; ++t) xJ[t * kScreenTile + tid] = xj[t];
        __syncthreads();  // s_c
        if (!valid) {
#pragma unroll
          for (int t = 0; t < KP; ++t) xj[t] = s_c[t];  // centred to zero
        }
        float cj[KP];
#pragma unroll
        for (int t = 0; t < KP; ++t) cj[t] = s_c[t];
        mj = build_row<KP>(xj, cj, tid, opB);
      } else {
        __syncthreads();  // s_c
        mj = build_row_xt<KP>(p.xt, p.npad, J * kScreenTile + tid, valid, s_c, tid, opB);
      }
      const bool bad = valid && !(mj < 1e30f);
      const int any_bad = __syncthreads_or(bad);
      put_ext(opB, tid, d, false, valid && !any_bad ? col_slack(mj, se) : 1e30f);
      if (tid == 0) s_badJ = any_bad;
      curJ = J;
    }

    // ---- operand A, in place of the stage ----
    const bool valid_i = tid < rows_i;
    if (!valid_i) {
#pragma unroll
      for (int t = 0; t < KP; ++t) xr[t] = s_c[t];  // centred to zero
    }
    float ci[KP];
#pragma unroll
    for (int t = 0; t < KP; ++t) ci[t] = s_c[t];
    const float nrow = build_row<KP>(xr, ci, tid, opA);
    const bool bad_i = valid_i && !(nrow < 1e30f);
    put_ext(opA, tid, d, true, valid_i && !bad_i ? row_slack(nrow, se) : 1e30f);
    fence_proxy_async_smem();
    tc_fence_before();
    const bool skip = __syncthreads_or(bad_i) || s_badJ;
    // the next item's tile I goes into the operand-A buffer once nothing reads it any more:
    // right away when this item issues no MMA, else when the MMA has completed
    auto stage_next = [&]() {
      if (e_nxt >= 0) {
        mbar_arrive_expect_tx(&bar_tma, kStageBytes);
        tma_load_2d(opA, &xt_map, static_cast<int32_t>((e_nxt & 0xffffffffLL) * kScreenTile), 0, &bar_tma);
        tma_pending = true;
      }
    };
    if (tid == 0) {
      publish();
      s_cnt[par ^ 1] = 0;  // the previous item's count: every thread has read it
      s_hits[par] = 0;     // this item's queue: flushed during the previous item
      if (skip) {
        // coordinates too large for the bound's arithmetic: exact tile kernel
        p.fallback[atomicAdd(p.counters + 5, 1ULL)] = e_cur;
        stage_next();
      } else {
        tc_fence_after();
        const uint32_t a0 = smem_u32(opA), b0 = smem_u32(opB);
#pragma unroll
        for (int s = 0; s < KS; ++s)
          umma_tf32(tmem, smem_desc_kmajor(a0 + s * kKStepBytes), smem_desc_kmajor(b0 + s * kKStepBytes), s > 0);
        umma_commit(&bar_mma);
      }
    }
    flush(par ^ 1);  // the previous item's pairs, while the MMA runs
    if (!skip) {
      const bool ok = mbar_wait_bounded(&bar_mma, ph_mma, kScreenPolls);
      if (tid == 0 && ok) stage_next();
      if (__syncthreads_or(!ok)) {
        failed = true;
        break;
      }
      ph_mma ^= 1u;
      tc_fence_after();

      // ---- screen: row tid of V, kLdCols columns per TMEM load ----
      uint32_t mask[4];
#pragma unroll
      for (int hh = 0; hh < 128 / kLdCols; ++hh) {
        uint32_t v[kLdCols];
        tmem_ld(trow + hh * kLdCols, v);
#pragma unroll
        for (int c2 = 0; c2 < kLdCols / 32; ++c2) {
          const int cc = hh * (kLdCols / 32) + c2;
          uint32_t all = 0xffffffffu;
#pragma unroll
          for (int j = 0; j < 32; ++j) all &= v[c2 * 32 + j];
          uint32_t hits = 0;
          if (!(all >> 31)) {
#pragma unroll
            for (int j = 0; j < 32; ++j) hits |= ((~v[c2 * 32 + j]) >> 31) << j;
            if (diag) {
              // strict upper triangle of the diagonal tile: columns > tid
              const int lo = tid - cc * 32;  // keep columns cc*32 + j with j > lo
              hits &= lo >= 31 ? 0u : (lo < 0 ? 0xffffffffu : (0xffffffffu << (lo + 1)));
            }
          }
          mask[cc] = hits;
        }
      }
      tc_fence_before();
      const int cnt = __popc(mask[0]) + __popc(mask[1]) + __popc(mask[2]) + __popc(mask[3]);
      if (cnt) atomicAdd(&s_cnt[par], cnt);
      __syncthreads();
      const int total = s_cnt[par];
      my_screened += 1;
      my_candidates += static_cast<unsigned long long>(total);
      if (total > (kSmemJ ? kScreenCap : kScreenCapXT)) {
        if (tid == 0) p.fallback[atomicAdd(p.counters + 5, 1ULL)] = e_cur;
      } else if (total > 0) {
        // ---- exact chain for each candidate of this row ----
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t hits = valid_i ? mask[cc] : 0u;
          while (hits) {
            const int j = cc * 32 + __ffs(hits) - 1;
            hits &= hits - 1;
            if (j >= cols_j) continue;
            // rows t >= d are 0 on both sides: fma(0, 0, w) == w, so the chain over KP rows
            // is bit-identical to the chain over d
            float w = 0.0f;
            const float* qj = p.xt + J * kScreenTile + j;
#pragma unroll
            for (int t = 0; t < KP; ++t) {
              const float xjt = kSmemJ ? xJ[t * kScreenTile + j] : __ldg(qj + t * p.npad);
              const float diff = __fsub_rn(xr[t], xjt);
              w = __fmaf_rn(diff, diff, w);
            }
            if (w <= cutoff && keep_pair(I * kScreenTile + tid, J * kScreenTile + j, p.keep_lo, p.keep_hi)) {
              int code = 0;
              while (w > s_eps2[code]) ++code;
              const int q = atomicAdd(&s_hits[par], 1);
              hitq[par * kScreenCap + q] = (static_cast<uint32_t>(code) << 28) | (static_cast<uint32_t>(tid) << 8) | static_cast<uint32_t>(j);
            }
          }
        }
      }
    }
    // ---- advance the item stream ----
    prev_row0 = static_cast<int32_t>(I) * kScreenTile;
    prev_col0 = static_cast<int32_t>(J) * kScreenTile;
    e_cur = e_nxt;
    e_nxt = e_nn;
    par ^= 1;
    if (++pos == clen) {
      if (tid == 0) grab(m & 1);
      ++m;
      cstart = s_chunk[m & 1];
      clen = s_clen[m & 1];
      pos = 0;
    }
  }

  if (!failed) {
    __syncthreads();  // the last item's queue is complete
    flush(par ^ 1);
  }
  if (failed) {
    if (tid == 0) atomicOr(p.err, kErrTmaTimeout);
    mbar_wait_bounded(&bar_mma, ph_mma, kScreenPolls);  // a bounded chance for the MMA to land
  }
  if (tid == 0 && tma_pending) mbar_wait_bounded(&bar_tma, ph_tma, kScreenPolls);  // and the stage load
  if (tid == 0) {
    if (my_candidates) atomicAdd(p.counters + 6, my_candidates);
    if (my_screened) atomicAdd(p.counters + 7, my_screened);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ---- host side ----------------------------------------------------------------------------------

bool screen_supported(int32_t d, float eps2_max)
{
  return d >= 1 && d <= 64 && eps2_max >= 1e-20f && eps2_max < 1e30f;
}

int32_t screen_rows(int32_t d) { return (d + 4 + 7) / 8 * 8; }

static size_t screen_smem_bytes(int ks, int32_t d)
{
  (void)d;
  const size_t xj = ks <= 5 ? static_cast<size_t>(8 * ks) * kScreenTile * sizeof(float) : 0;  // kSmemJ
  const size_t need = 1024 + static_cast<size_t>(2 * ks) * kKStepBytes + xj + 2 * kScreenCap * sizeof(uint32_t);
  return need < kScreenMinSmem ? kScreenMinSmem : need;
}

template <int KS>
static Status launch_screen_ks(const ScreenParams& p, int sm_count, cudaStream_t s)
{
  CUtensorMap map;
  DBM_TRY(make_tile_map(p.xt, p.n, 8 * KS, &map));
  const size_t smem = screen_smem_bytes(KS, p.d);
  DBM_CUDA(cudaFuncSetAttribute(dist_screen_kernel<KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  DBM_CUDA(cudaFuncSetAttribute(dist_screen_kernel<KS>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared));
  // CTAs per SM from the device's shared-memory and register limits (the occupancy query
  // reports one CTA for kernels that allocate tensor memory); never more than 4, so that
  // 4 x 128 TMEM columns always fit and no tcgen05.alloc can wait.
  cudaFuncAttributes fa{};
  DBM_CUDA(cudaFuncGetAttributes(&fa, dist_screen_kernel<KS>));
  int dev = 0, smem_sm = 0, smem_rsv = 0, regs_sm = 0;
  DBM_CUDA(cudaGetDevice(&dev));
  DBM_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
  DBM_CUDA(cudaDeviceGetAttribute(&smem_rsv, cudaDevAttrReservedSharedMemoryPerBlock, dev));
  DBM_CUDA(cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev));
  const int regs_warp = (std::max(fa.numRegs, 1) * 32 + 255) / 256 * 256;
  const int by_regs = regs_sm / (regs_warp * (kScreenThreads / 32));
  const int by_smem = smem_sm / static_cast<int>(smem + fa.sharedSizeBytes + smem_rsv);
  int per_sm = std::min(std::min(by_regs, by_smem), 4);
  if (per_sm < 1) per_sm = 1;
  int64_t grid = static_cast<int64_t>(sm_count) * per_sm;
  const int64_t chunks = ceil_div(p.item_count, kScreenGrab);
  if (grid > chunks) grid = chunks;
  if (grid < 1) return Status::Ok();
  count_launch();
  dist_screen_kernel<KS><<<static_cast<unsigned>(grid), kScreenThreads, smem, s>>>(map, p);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

Status launch_screened_distance(const DistLaunch& a, const float* box_lo, const float* box_hi, long long* fallback,
                                cudaStream_t s)
{
  if (!a.work || !a.perm) return Status::Err(DBM_ERR_INVALID, "screened distance pass needs a worklist");
  if (!screen_supported(a.d, a.eps2[a.k - 1])) return Status::Err(DBM_ERR_INVALID, "screened distance pass needs D <= 64");
  ScreenParams p{};
  p.n = a.n;
  p.npad = (a.n + 3) / 4 * 4;
  p.d = a.d;
  p.k = a.k;
  const int shards = a.nshards > 0 ? a.nshards : 1;
  p.shard = a.shard;
  p.nshards = shards;
  if (a.work_total_dev) {
    p.total_dev = a.work_total_dev;
    p.cap = a.work_cap;
    p.item_count = a.work_cap;  // an upper bound for the grid size
  } else {
    p.item_count = shard_items(a.work_count, a.shard, shards);
  }
  p.work = a.work;
  p.xt = a.xt;
  p.counters = a.counters;
  p.edges = a.edges;
  p.edge_cap = a.edge_cap;
  p.hist = a.hist;
  p.err = a.err;
  p.perm = a.perm;
  p.box_lo = box_lo;
  p.box_hi = box_hi;
  p.tiles = ceil_div(a.n, kScreenTile);
  p.fallback = fallback;
  p.keep_lo = a.keep_lo;
  p.keep_hi = a.keep_hi;
  for (int e = 0; e < kMaxEps; ++e) p.eps2[e] = e < a.k ? a.eps2[e] : a.eps2[a.k - 1];
  {
    const double e = static_cast<double>(a.eps2[a.k - 1]) * (1.0 + (a.d + 3) * std::ldexp(1.0, -24));
    float sq = static_cast<float>(std::sqrt(e));
    while (static_cast<double>(sq) * sq < e) sq = std::nextafter(sq, INFINITY);
    p.sqrt_e = sq;
  }
  const int ks = (a.d + 4 + 7) / 8;
  switch (ks) {
    case 1: return launch_screen_ks<1>(p, a.sm_count, s);
    case 2: return launch_screen_ks<2>(p, a.sm_count, s);
    case 3: return launch_screen_ks<3>(p, a.sm_count, s);
    case 4: return launch_screen_ks<4>(p, a.sm_count, s);
    case 5: return launch_screen_ks<5>(p, a.sm_count, s);
    case 6: return launch_screen_ks<6>(p, a.sm_count, s);
    case 7: return launch_screen_ks<7>(p, a.sm_count, s);
    case 8: return launch_screen_ks<8>(p, a.sm_count, s);
    case 9: return launch_screen_ks<9>(p, a.sm_count, s);
    default: return Status::Err(DBM_ERR_INVALID, "screened distance pass needs D <= 64");
  }
}

}  // namespace dbm
