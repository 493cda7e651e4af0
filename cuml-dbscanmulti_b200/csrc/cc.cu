// cc.cu -- batched connected components, cross-batch label merge and final relabel.
//
// What the reference computes (Math-BUG/cuML-DBSCANMulti, runner_multi.cuh:1045-1092 and
// 1228-1234, with RAFT's weak_cc_batched / merge_labels / make_monotonic): for each config,
// batches in ascending order, a weak-CC over the batch's rows with the core mask as filter
// (labels min-index + 1 per core component, non-core points take the smallest adjacent core
// label the batch can see), merged into the accumulated labels by a root map R, then ids by
// rank of the surviving labels.  The resulting labels have a closed form that these kernels
// evaluate directly, with one global union-find instead of a merge per batch:
//
//   core point c:   label = minimum index of c's core component (over every batch's edges);
//   border point p: cur(p) is folded batch by batch, b = 0..nb-1, as
//                     cur = min(G_b(cur), G_b(L_b*(p)))
//                   where G_b is the global union-find after batch b's edges, and L_b*(p) is the
//                   smallest batch-local component root among the core neighbours of p that
//                   batch b can see (edges whose row lies in batch b).  That is exactly the
//                   value RAFT's merge leaves in labels_a, including its dependence on the
//                   batch partition and order for points adjacent to several clusters.
//
// Everything is min-index union-find: roots are hooked larger-under-smaller with atomicCAS,
// so a root is always its tree's minimum and the fixpoint does not depend on thread order.
// Per-(batch, eps) kernels process the l minPts configs of that eps together: with minPts
// ascending, a point is core for config (e, m) iff m < corecnt[e][i].
#include "dbm_internal.cuh"

#include <algorithm>

namespace dbm {


// Layout of the forests (G, L), the border candidates (best) and the folded labels (cur): the l
// configs of an eps are interleaved point by point, config (e, m) of point i at element
// (e n + i) l + m = fbase(e, m) + i l.  An entry's per-config gathers and union-find steps for
// one point then share a 32-byte sector instead of touching l arrays n elements apart (C4
// labelling -10%, C1 -25% against one array per config; the calibrated dense C5 is unchanged).
__host__ __device__ __forceinline__ int64_t fbase(int64_t n, int l, int e, int m)
{
  return static_cast<int64_t>(e) * n * l + m;
}

__global__ void cc_init_kernel(int64_t n, int l, int64_t total, int32_t* __restrict__ G,
                               int32_t* __restrict__ cur, unsigned long long* __restrict__ best)
{
  const int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (x >= total) return;
  G[x] = static_cast<int32_t>((x / l) % n);
  cur[x] = kNone;
  best[x] = ~0ull;
}

// ---- one batch, all eps at once ---------------------------------------------------------------
// Each kernel walks every neighbour entry of the batch's rows once per eps it belongs to and does
// its work for the minPts configs of that eps that this call owns ([cfg_begin, cfg_end)):
//   annotated route: slab e holds the entries of eps e (compacted), e = 0..k-1;
//   direct route:    slab 0 holds the max-eps entries with their codes (col >> 28), and an
//                    entry belongs to every eps e >= its code (no per-eps copies).
struct CcArgs {
  MultiSlab ms;
  int64_t n;
  int k, l, cfg_begin, cfg_end;
  const int32_t* cc;  // k x n: core iff m < cc[e*n + i]
  const uint8_t* cc8 = nullptr;  // the same counts as bytes (l <= 255), read by the entry walks
  int sample_shift = 0;  // union over every 2^s-th entry only (0: all entries)
  bool quick = false;    // union: skip a union-find whose two endpoints already share a parent
  int union_limit = kUnionRetryLimit;  // retry bound of each uf_unite (lowered only by a test knob)
};

// core count of point x at eps e: the byte copy when there is one (its k x n bytes stay in L1/L2
// far better than the int32 array under the random gathers of an entry walk)
__device__ __forceinline__ int core_count(const CcArgs& a, int e, int32_t x)
{
  const int64_t at = static_cast<int64_t>(e) * a.n + x;
  return a.cc8 ? static_cast<int>(__ldg(a.cc8 + at)) : __ldg(a.cc + at);
}

__device__ __forceinline__ void cfg_range(const CcArgs& a, int e, int& m_lo, int& m_hi)
{
  m_lo = max(0, min(a.l, a.cfg_begin - e * a.l));
  m_hi = max(0, min(a.l, a.cfg_end - e * a.l));
}

template <class F>
__device__ __forceinline__ void for_each_entry(const CcArgs& a, F&& f)
{
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (a.ms.direct) {
    const SlabRef& s = a.ms.s[0];
    for (int64_t q = t0; q < s.count; q += stride) {
      const uint32_t w = static_cast<uint32_t>(s.col[q]);
      const int32_t j = static_cast<int32_t>(w & kColMask);
      const int e0 = max(static_cast<int>(w >> kCodeShift), a.cfg_begin / a.l);
      const int e1 = min(a.k, (a.cfg_end + a.l - 1) / a.l);  // owned eps [e0, e1)
      if (e0 >= e1) continue;  // beyond every owned eps: the row index is not even read
      const int32_t r = s.row[q];
      for (int e = e0; e < e1; ++e) f(e, r, j);
    }
  } else {
    for (int e = 0; e < a.ms.nslabs; ++e) {
      int m_lo, m_hi;
      cfg_range(a, e, m_lo, m_hi);
      if (m_lo >= m_hi) continue;  // no config of this eps is owned by this call
      const SlabRef& s = a.ms.s[e];
      const int64_t b = s.begin_dev ? *s.begin_dev : 0;
      const int64_t lim = s.end_dev ? *s.end_dev : s.count;
      for (int64_t q = b + t0; q < lim; q += stride) f(e, s.row[q], s.col[q] & static_cast<int32_t>(kColMask));
    }
  }
}

// One thread per (entry, minPts index m), for the union kernel: the union-find chains of the l
// configs of an entry are independent, so giving each its own thread keeps l times more memory
// requests in flight (the kernel is bound by the latency of dependent L2 accesses, not by
// bandwidth).  The lighter kernels (one find or store per config) keep one thread per entry.  f(e, m, r, j)
// runs for every eps e the entry belongs to and every m of e owned by this call.
// The flat index x = entry * span + m walks the grid-stride loop as the pair (entry, m), advanced
// by the stride's own quotient and remainder (two divisions per thread, none per item: a 64-bit
// division per item made the dense-graph union instruction-bound).
struct FlatCursor {
  int64_t q, dq;  // entry index and its step
  int m, dm;      // minPts index and its step
  __device__ __forceinline__ FlatCursor(int64_t t0, int64_t stride, int span)
  {
    q = t0 / span;
    m = static_cast<int>(t0 - q * span);
    dq = stride / span;
    dm = static_cast<int>(stride - dq * span);
  }
  __device__ __forceinline__ void advance(int span)
  {
    q += dq;
    m += dm;
    if (m >= span) {
      m -= span;
      q += 1;
    }
  }
};

template <class F>
__device__ __forceinline__ void for_each_entry_cfg(const CcArgs& a, F&& f)
{
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int L = a.l;
  const int sh = a.sample_shift;
  if (a.ms.direct) {
    const SlabRef& s = a.ms.s[0];
    const int64_t entries = (s.count + (int64_t(1) << sh) - 1) >> sh;
    for (FlatCursor c(t0, stride, L); c.q < entries; c.advance(L)) {
      const int m = c.m;
      const int64_t q = c.q << sh;
      const uint32_t w = static_cast<uint32_t>(s.col[q]);
      const int32_t j = static_cast<int32_t>(w & kColMask);
      const int e0 = max(static_cast<int>(w >> kCodeShift), a.cfg_begin / a.l);
      const int e1 = min(a.k, (a.cfg_end + a.l - 1) / a.l);  // owned eps [e0, e1)
      if (e0 >= e1) continue;
      const int32_t r = s.row[q];
      for (int e = e0; e < e1; ++e) {
        int m_lo, m_hi;
        cfg_range(a, e, m_lo, m_hi);
        if (m >= m_lo && m < m_hi) f(e, m, r, j);
      }
    }
  } else {
    for (int e = 0; e < a.ms.nslabs; ++e) {
      int m_lo, m_hi;
      cfg_range(a, e, m_lo, m_hi);
      if (m_lo >= m_hi) continue;  // no config of this eps is owned by this call
      const SlabRef& s = a.ms.s[e];
      const int64_t b = s.begin_dev ? *s.begin_dev : 0;
      const int64_t lim = s.end_dev ? *s.end_dev : s.count;
      const int span = m_hi - m_lo;
      const int64_t entries = (lim - b + (int64_t(1) << sh) - 1) >> sh;
      for (FlatCursor c(t0, stride, span); c.q < entries; c.advance(span)) {
        const int64_t q = b + (c.q << sh);
        f(e, m_lo + c.m, s.row[q], s.col[q] & static_cast<int32_t>(kColMask));
      }
    }
  }
}

// L[cfg][v] = v for both endpoints of every entry (configs where v is core).
__global__ void cc_touch_kernel(const CcArgs a, int32_t* __restrict__ L)
{
  for_each_entry(a, [&](int e, int32_t r, int32_t j) {
    int m_lo, m_hi;
    cfg_range(a, e, m_lo, m_hi);
    const int cr = min(core_count(a, e, r), m_hi), cj = min(core_count(a, e, j), m_hi);
    for (int m = m_lo; m < cr; ++m) L[fbase(a.n, a.l, e, m) + static_cast<int64_t>(r) * a.l] = r;
    for (int m = m_lo; m < cj; ++m) L[fbase(a.n, a.l, e, m) + static_cast<int64_t>(j) * a.l] = j;
  });
}

// unite(P[cfg], r, j) for every core-core entry; with Q set, unite(Q[cfg], r, j) as well (the
// batch-local and the global union-find of a batch share one walk of its entries)
__global__ void cc_union_kernel(const CcArgs a, int32_t* __restrict__ P, int32_t* __restrict__ Q,
                                int32_t* __restrict__ err)
{
  bool ok = true;
  for_each_entry_cfg(a, [&](int e, int m, int32_t r, int32_t j) {
    const int64_t base = fbase(a.n, a.l, e, m);
    const int64_t pr = base + static_cast<int64_t>(r) * a.l, pj = base + static_cast<int64_t>(j) * a.l;
    // the core counts are read together with the parents (one round of memory latency, not two)
    const int cr = core_count(a, e, r), cj = core_count(a, e, j);
    // equal parents mean the union is a no-op, exact whatever the state of the forest (a stale
    // batch-local parent of a non-core endpoint can only skip a union the core test below would
    // skip too); after a compression most endpoint pairs of one component take this exit
    const bool skip_p = a.quick && P[pr] == P[pj];
    const bool skip_q = !Q || (a.quick && Q[pr] == Q[pj]);
    if (skip_p && skip_q) return;
    if (m >= cr || m >= cj) return;
    if (!skip_p) ok &= uf_unite(P + base, r, j, a.union_limit, a.l);
    if (!skip_q) ok &= uf_unite(Q + base, r, j, a.union_limit, a.l);
  });
  if (!ok) atomicOr(err, kErrUnionLimit);
}

// P[x] = x for every x of the configs [c0, c1): a fresh forest (the batch-local one of a dense
// batch, which is then compressed over every point and so must hold no stale parents from an
// earlier batch or fit)
__global__ void cc_reset_kernel(int64_t n, int l, int c0, int c1, int32_t* __restrict__ P)
{
  const int64_t total = static_cast<int64_t>(c1 - c0) * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < total; x += stride) {
    const int64_t cfg = c0 + x / n, i = x % n;
    P[fbase(n, l, static_cast<int>(cfg / l), static_cast<int>(cfg % l)) + i * l] = static_cast<int32_t>(i);
  }
}

// Root snapshot of a dense batch: per eps e and point x, kSnapSlots int32 -- slots 0-3 the roots
// of x in the union's first forest for minPts index m = 0..3, slots 4-7 in its second forest.
constexpr int kSnapSlots = 8;
constexpr int kSnapConfigs = 4;

// P[x] = root of x for every x of the configs [c0, c1) (full path compression); with R set, the
// roots also go to slot `slot + m` of R (configs with m < 4)
__global__ void cc_compress_kernel(int64_t n, int l, int c0, int c1, int32_t* __restrict__ P,
                                   int32_t* __restrict__ R, int slot)
{
  const int64_t total = static_cast<int64_t>(c1 - c0) * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < total; x += stride) {
    const int64_t cfg = c0 + x / n, i = x % n;
    const int e = static_cast<int>(cfg / l), m = static_cast<int>(cfg % l);
    int32_t* g = P + fbase(n, l, e, m);
    const int32_t root = uf_find(g, static_cast<int32_t>(i), l);
    if (g[i * l] != root) g[i * l] = root;
    if (R && m < kSnapConfigs) R[(static_cast<int64_t>(e) * n + i) * kSnapSlots + slot + m] = root;
  }
}

__device__ __forceinline__ unsigned eq_roots(const int4& a, const int4& b)
{
  return static_cast<unsigned>(a.x == b.x) | (static_cast<unsigned>(a.y == b.y) << 1) |
         (static_cast<unsigned>(a.z == b.z) << 2) | (static_cast<unsigned>(a.w == b.w) << 3);
}

// The full union pass of a dense batch after the sampled pass and the compression: one thread
// per entry, U entries in flight per thread.  Both endpoints under one snapshot root (R) make
// the union a no-op in that forest, since forests only merge; so a typical entry costs one
// 32-byte load of its column point's roots (the row point's are shared by the warp) instead of
// two gathers per config and forest.  Entries still open go through the forests as usual.
// P: the forest of slots 0-3; Q (optional): slots 4-7.
template <int U>
__global__ void __launch_bounds__(256) cc_union_snap_kernel(const CcArgs a, int32_t* __restrict__ P,
                                                            int32_t* __restrict__ Q,
                                                            const int4* __restrict__ R, int32_t* __restrict__ err)
{
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int e_lo = a.cfg_begin / a.l, e_hi = min(a.k, (a.cfg_end + a.l - 1) / a.l);
  bool ok = true;
  for (int e = e_lo; e < e_hi; ++e) {
    int m_lo, m_hi;
    cfg_range(a, e, m_lo, m_hi);
    if (m_lo >= m_hi) continue;
    // direct route: every eps walks the max-eps slab and keeps the entries of code <= e
    const SlabRef& s = a.ms.direct ? a.ms.s[0] : a.ms.s[e];
    if (!a.ms.direct && e >= a.ms.nslabs) continue;
    const int64_t b = s.begin_dev ? *s.begin_dev : 0;
    const int64_t lim = s.end_dev ? *s.end_dev : s.count;
    const int m4 = min(m_hi, kSnapConfigs);
    const unsigned owned4 = m_lo < m4 ? ((1u << m4) - 1u) & ~((1u << m_lo) - 1u) : 0u;
    const bool tail = m_hi > kSnapConfigs;  // configs without a snapshot: always through the forests
    const int4* Re = R + static_cast<int64_t>(e) * a.n * 2;
    for (int64_t q0 = b + t0; q0 < lim; q0 += U * stride) {
      int32_t r[U], j[U];
      bool v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t q = q0 + u * stride;
        v[u] = q < lim;
        const uint32_t w = v[u] ? static_cast<uint32_t>(s.col[q]) : 0u;
        r[u] = v[u] ? s.row[q] : 0;
        j[u] = static_cast<int32_t>(w & kColMask);
        if (a.ms.direct) v[u] = v[u] && static_cast<int>(w >> kCodeShift) <= e;
      }
      int4 pr[U], pj[U], qr[U], qj[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (!v[u]) continue;
        pr[u] = Re[2 * static_cast<int64_t>(r[u])];
        pj[u] = Re[2 * static_cast<int64_t>(j[u])];
        if (Q) {
          qr[u] = Re[2 * static_cast<int64_t>(r[u]) + 1];
          qj[u] = Re[2 * static_cast<int64_t>(j[u]) + 1];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (!v[u]) continue;
        const unsigned open_p = owned4 & ~eq_roots(pr[u], pj[u]);
        const unsigned open_q = Q ? owned4 & ~eq_roots(qr[u], qj[u]) : 0u;
        if (!tail && !(open_p | open_q)) continue;
        const int core_hi = min(m_hi, min(core_count(a, e, r[u]), core_count(a, e, j[u])));
        for (int m = m_lo; m < core_hi; ++m) {
          const int64_t base = fbase(a.n, a.l, e, m);
          const bool snap = m < kSnapConfigs;
          if (!snap || ((open_p >> m) & 1u)) ok &= uf_unite(P + base, r[u], j[u], a.union_limit, a.l);
          if (Q && (!snap || ((open_q >> m) & 1u))) ok &= uf_unite(Q + base, r[u], j[u], a.union_limit, a.l);
        }
      }
    }
  }
  if (!ok) atomicOr(err, kErrUnionLimit);
}

// For every entry with exactly one core endpoint c: best[p] = min(tag << 32 | find(P, c)).
__global__ void cc_best_kernel(const CcArgs a, int32_t* __restrict__ P, unsigned long long* __restrict__ best,
                               uint32_t tag)
{
  for_each_entry(a, [&](int e, int32_t r, int32_t j) {
    int m_lo, m_hi;
    cfg_range(a, e, m_lo, m_hi);
    const int cr = core_count(a, e, r), cj = core_count(a, e, j);
    const int lo = max(min(cr, cj), m_lo), hi = min(max(cr, cj), m_hi);
    for (int m = lo; m < hi; ++m) {
      const bool r_core = m < cr;
      const int32_t c = r_core ? r : j;
      const int32_t pt = r_core ? j : r;
      const int64_t base = fbase(a.n, a.l, e, m);
      const int32_t root = uf_find(P + base, c, a.l);
      atomicMin(best + base + static_cast<int64_t>(pt) * a.l,
                (static_cast<unsigned long long>(tag) << 32) | static_cast<uint32_t>(root));
    }
  });
}

// cur[p] = min(find(G, cur[p]), find(G, best[p])) for every border endpoint.
__global__ void cc_border_kernel(const CcArgs a, int32_t* __restrict__ G,
                                 const unsigned long long* __restrict__ best, int32_t* __restrict__ cur,
                                 uint32_t tag)
{
  for_each_entry(a, [&](int e, int32_t r, int32_t j) {
    int m_lo, m_hi;
    cfg_range(a, e, m_lo, m_hi);
    const int cr = core_count(a, e, r), cj = core_count(a, e, j);
    const int lo = max(min(cr, cj), m_lo), hi = min(max(cr, cj), m_hi);
    for (int m = lo; m < hi; ++m) {
      const int32_t pt = (m < cr) ? j : r;
      const int64_t base = fbase(a.n, a.l, e, m);
      const int64_t at = base + static_cast<int64_t>(pt) * a.l;
      const unsigned long long v = best[at];
      if (static_cast<uint32_t>(v >> 32) != tag) continue;
      const int32_t cand = uf_find(G + base, static_cast<int32_t>(v & 0xffffffffu), a.l);
      volatile int32_t* cp = cur + at;
      const int32_t old = *cp;
      const int32_t prev = (old == kNone) ? kNone : uf_find(G + base, old, a.l);
      *cp = prev < cand ? prev : cand;
    }
  });
}

// The same fold per point rather than per entry, for batches with many more entries than
// points x configs: best[p] carries this batch's tag iff some entry of the batch gave p a border
// candidate, and every such entry folds the same value into cur[p].
__global__ void cc_border_points_kernel(int64_t n, int l, int c0, int c1, const int32_t* __restrict__ cc,
                                        int32_t* __restrict__ G, const unsigned long long* __restrict__ best,
                                        int32_t* __restrict__ cur, uint32_t tag)
{
  const int64_t total = static_cast<int64_t>(c1 - c0) * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < total; x += stride) {
    const int64_t cfg = c0 + x / n, i = x - (cfg - c0) * n;
    const int e = static_cast<int>(cfg / l), m = static_cast<int>(cfg % l);
    const int64_t base = fbase(n, l, e, m), at = base + i * l;
    const unsigned long long v = best[at];
    if (static_cast<uint32_t>(v >> 32) != tag) continue;
    if (m < cc[static_cast<int64_t>(e) * n + i]) continue;  // core points take no border candidate
    int32_t* g = G + base;
    const int32_t cand = uf_find(g, static_cast<int32_t>(v & 0xffffffffu), l);
    const int32_t old = cur[at];
    const int32_t prev = (old == kNone) ? kNone : uf_find(g, old, l);
    cur[at] = prev < cand ? prev : cand;
  }
}

// Roots of the configs [c0, c1) as a bitmap: config cfg owns W = ceil(n / 32) words, bit i of its
// word i / 32 is set iff i is the root (minimum index) of a core component; cnt[w - c0 * W] is the
// popcount of word w.  One thread per (config, padded point), so every warp covers one whole word.
__global__ void cc_root_bits_kernel(int64_t n, int l, int c0, int c1, int64_t W, const int32_t* __restrict__ cc,
                                    int32_t* __restrict__ G, uint32_t* __restrict__ words, int32_t* __restrict__ cnt)
{
  const int64_t per = W * 32;
  const int64_t total = static_cast<int64_t>(c1 - c0) * per;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;  // a multiple of 32
  for (int64_t x = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; x < total; x += stride) {
    const int64_t cl = x / per, i = x - cl * per, cfg = c0 + cl;
    const int e = static_cast<int>(cfg / l), m = static_cast<int>(cfg % l);
    bool root = false;
    if (i < n && m < cc[static_cast<int64_t>(e) * n + i])
      root = uf_find(G + fbase(n, l, e, m), static_cast<int32_t>(i), l) == static_cast<int32_t>(i);
    const uint32_t bits = __ballot_sync(0xffffffffu, root);
    if ((threadIdx.x & 31) == 0) {
      const int64_t w = cl * W + i / 32;
      words[c0 * W + w] = bits;
      cnt[w] = __popc(bits);
    }
  }
}

// cluster id = rank of the component root among the config's roots (word prefix from the scan of
// the popcounts, plus the set bits below the root in its word); -1 noise
__global__ void cc_labels_kernel(int64_t n, int l, int c0, int c1, int64_t W, const int32_t* __restrict__ cc,
                                 int32_t* __restrict__ G, const int32_t* __restrict__ cur,
                                 const uint32_t* __restrict__ words, const int64_t* __restrict__ wrank,
                                 int32_t* __restrict__ labels)
{
  // threads in the forests' interleaved order (point-major within an eps, minPts config
  // fastest): the parent and folded-label reads of a warp are contiguous, and its label writes
  // are l runs of 32 / l consecutive points
  const int e0 = c0 / l;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t per_eps = n * l;
  const int e = e0 + static_cast<int>(t / per_eps);
  const int64_t rem = t - static_cast<int64_t>(e - e0) * per_eps;
  const int64_t i = rem / l;
  const int m = static_cast<int>(rem - i * l);
  const int64_t cfg = static_cast<int64_t>(e) * l + m;
  if (cfg < c0 || cfg >= c1) return;
  const int64_t x = cfg * n + i;
  int32_t* g = G + fbase(n, l, e, m);
  int32_t v;
  if (m < cc[static_cast<int64_t>(e) * n + i]) {
    v = static_cast<int32_t>(i);
  } else {
    v = cur[fbase(n, l, e, m) + i * l];
    if (v == kNone) {
      labels[x] = -1;
      return;
    }
  }
  const int32_t root = uf_find(g, v, l);
  const int64_t wl = (cfg - c0) * W;  // this config's first word in the scanned range
  const int64_t w = wl + root / 32;
  const uint32_t below = words[cfg * W + root / 32] & ((1u << (root & 31)) - 1u);
  labels[x] = static_cast<int32_t>(wrank[w] - wrank[wl]) + __popc(below);
}

// ---- launchers ----------------------------------------------------------------------------
static inline unsigned blocks_for(int64_t work, int threads)
{
  return static_cast<unsigned>(ceil_div(work > 0 ? work : 1, threads));
}

Status launch_cc_init(int64_t n, int k, int l, int32_t* G, int32_t* cur, unsigned long long* best,
                      cudaStream_t s)
{
  const int64_t total = n * k * l;
  count_launch();
  cc_init_kernel<<<blocks_for(total, 256), 256, 0, s>>>(n, l, total, G, cur, best);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

// One batch, every eps: local components (when there is more than one batch), border
// candidates, global union, border fold.
Status launch_cc_batch(const MultiSlab& ms, int64_t upper_entries, int64_t n, int64_t rows, int k, int l,
                       int cfg_begin, int cfg_end, const int32_t* cc, const uint8_t* cc8, bool single_batch,
                       int32_t* G, int32_t* L,
                       unsigned long long* best, int32_t* cur, uint32_t tag, int32_t* err, int sm_count,
                       int union_limit, int32_t* snap, cudaStream_t s)
{
  if (upper_entries <= 0 || cfg_begin >= cfg_end) return Status::Ok();
  CcArgs a{ms, n, k, l, cfg_begin, cfg_end, cc};
  a.cc8 = cc8;
  a.quick = true;
  a.union_limit = union_limit;
  const unsigned nb = static_cast<unsigned>(
    std::max<int64_t>(1, std::min<int64_t>(ceil_div(upper_entries, 256), static_cast<int64_t>(sm_count) * 16)));
  const unsigned nbu = static_cast<unsigned>(
    std::max<int64_t>(1, std::min<int64_t>(ceil_div(upper_entries * l, 256), static_cast<int64_t>(sm_count) * 32)));
  // dense batches (afforest-style sampling, Sutton et al. 2018): unite a 1/16 sample of the
  // entries, compress (recording every point's roots in `snap`), then the full pass finds most
  // endpoint pairs already under one snapshot root and skips them; the forests' roots are the
  // same as a plain pass would leave
  CcArgs sa = a;
  sa.sample_shift = 4;  // 1/16: calibrated dense C5 labelling 247 ms (1/8: 288 ms, 1/4: 385 ms, 1/64: 305 ms)
  const unsigned nbs = static_cast<unsigned>(std::max<int64_t>(
    1, std::min<int64_t>(ceil_div((upper_entries >> sa.sample_shift) * l, 256), static_cast<int64_t>(sm_count) * 32)));
  const unsigned nbc = static_cast<unsigned>(std::max<int64_t>(
    1, std::min<int64_t>(ceil_div(static_cast<int64_t>(cfg_end - cfg_begin) * n, 256), static_cast<int64_t>(sm_count) * 16)));
  // entries in flight per thread of the snapshot union: 1 measured fastest (calibrated dense C5
  // labelling 271 ms, against 361 ms with 2 and 319 ms with 4: the unrolled forms hold more
  // registers and lose more occupancy than the extra loads in flight win back)
  constexpr int kSnapUnroll = 1;
  const unsigned nbe = static_cast<unsigned>(std::max<int64_t>(
    1, std::min<int64_t>(ceil_div(upper_entries, 256 * kSnapUnroll), static_cast<int64_t>(sm_count) * 32)));
  if (single_batch && upper_entries >= kDenseEntriesPerRow * n) {
    count_launch(4);
    cc_union_kernel<<<nbs, 256, 0, s>>>(sa, G, nullptr, err);
    cc_compress_kernel<<<nbc, 256, 0, s>>>(n, l, cfg_begin, cfg_end, G, snap, 0);
    if (snap)
      cc_union_snap_kernel<kSnapUnroll><<<nbe, 256, 0, s>>>(a, G, nullptr, reinterpret_cast<const int4*>(snap), err);
    else
      cc_union_kernel<<<nbu, 256, 0, s>>>(a, G, nullptr, err);
    cc_best_kernel<<<nb, 256, 0, s>>>(a, G, best, tag);
  } else if (single_batch) {
    count_launch(2);
    cc_union_kernel<<<nbu, 256, 0, s>>>(a, G, nullptr, err);
    cc_best_kernel<<<nb, 256, 0, s>>>(a, G, best, tag);
  } else if (upper_entries >= kDenseEntriesPerRow * rows) {
    // a dense batch of a multi-batch fit: the same sampling for the batch-local and the global
    // forest at once, then the full union.  The batch-local forest is reset over the owned
    // configs (a superset of what cc_touch sets), because the compression walks every point's
    // chain and stale parents from earlier batches or fits need not be valid chains of this one;
    // the global forest holds only this fit's chains (cc_init).
    count_launch(6);
    cc_reset_kernel<<<nbc, 256, 0, s>>>(n, l, cfg_begin, cfg_end, L);
    cc_union_kernel<<<nbs, 256, 0, s>>>(sa, L, G, err);
    cc_compress_kernel<<<nbc, 256, 0, s>>>(n, l, cfg_begin, cfg_end, L, snap, 0);
    cc_compress_kernel<<<nbc, 256, 0, s>>>(n, l, cfg_begin, cfg_end, G, snap, kSnapConfigs);
    if (snap)
      cc_union_snap_kernel<kSnapUnroll><<<nbe, 256, 0, s>>>(a, L, G, reinterpret_cast<const int4*>(snap), err);
    else
      cc_union_kernel<<<nbu, 256, 0, s>>>(a, L, G, err);
    cc_best_kernel<<<nb, 256, 0, s>>>(a, L, best, tag);
  } else {
    // the global union needs only to precede the border fold, so it rides along with the local
    // one; the border candidates read the finished local union-find
    count_launch(3);
    cc_touch_kernel<<<nb, 256, 0, s>>>(a, L);
    cc_union_kernel<<<nbu, 256, 0, s>>>(a, L, G, err);
    cc_best_kernel<<<nb, 256, 0, s>>>(a, L, best, tag);
  }
  count_launch();
  const int64_t cfg_points = static_cast<int64_t>(cfg_end - cfg_begin) * n;
  if (cfg_points <= upper_entries) {
    const unsigned nbp = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>(ceil_div(cfg_points, 256), static_cast<int64_t>(sm_count) * 16)));
    cc_border_points_kernel<<<nbp, 256, 0, s>>>(n, l, cfg_begin, cfg_end, cc, G, best, cur, tag);
  } else {
    cc_border_kernel<<<nb, 256, 0, s>>>(a, G, best, cur, tag);
  }
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

Status launch_cc_root_bits(int64_t n, int l, int c0, int c1, int64_t W, const int32_t* cc,
                           int32_t* G, uint32_t* words, int32_t* cnt, int sm_count, cudaStream_t s)
{
  const int64_t total = static_cast<int64_t>(c1 - c0) * W * 32;
  if (total <= 0) return Status::Ok();
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(
    1, std::min<int64_t>(ceil_div(total, 256), static_cast<int64_t>(sm_count) * 32)));
  count_launch();
  cc_root_bits_kernel<<<grid, 256, 0, s>>>(n, l, c0, c1, W, cc, G, words, cnt);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

Status launch_cc_labels(int64_t n, int l, int c0, int c1, int64_t W, const int32_t* cc, int32_t* G,
                        const int32_t* cur, const uint32_t* words, const int64_t* wrank, int32_t* labels,
                        cudaStream_t s)
{
  if (c1 <= c0) return Status::Ok();
  // every (point, config) of the eps the range touches; threads outside the range return
  const int64_t total = static_cast<int64_t>((c1 + l - 1) / l - c0 / l) * n * l;
  count_launch();
  cc_labels_kernel<<<blocks_for(total, 256), 256, 0, s>>>(n, l, c0, c1, W, cc, G,
                                                          cur, words, wrank, labels);
  DBM_CUDA(cudaGetLastError());
  return Status::Ok();
}

}  // namespace dbm
