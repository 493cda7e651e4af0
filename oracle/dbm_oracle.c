/*
 * dbm_oracle.c -- CPU restatement of the reference's multi-parameter DBSCAN (`fit_multi`).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA product path is
 * compared against; it is never linked into, loaded by, or called from the product library
 * (libdbm.so) or its Python host layer.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg may load it.
 *
 * What is restated, and where it comes from in the reference (Math-BUG/cuML-DBSCANMulti):
 *
 *  - pair arithmetic: src/multi/eps_neighborhood.cuh:151-158 -- `acc += diff*diff` over
 *    d = 0..D-1, which nvcc (default --fmad=true, Makefile:195-198) contracts to the
 *    sequential fused multiply-add acc = fma(x_i[d]-x_j[d], x_i[d]-x_j[d], acc).  Pairs are
 *    neighbours when acc <= eps2[e] (closed ball, the point itself included), with
 *    eps2 = eps*eps rounded to float on the host (src/main.cu:522-523).
 *  - per-pair code = smallest e with acc <= eps2[e], 255 when none
 *    (src/multi/eps_neighborhood.cuh:160-168); per-eps degree = #pairs with code <= e
 *    (src/multi/eps_neighborhood.cuh:171-174).
 *  - core masks: degree_e(i) >= minPts[m], eps-major config = e*l + m
 *    (src/multi/corepoints_multi.cuh:104-120).
 *  - batched labelling: for each row batch, RAFT weak_cc_batched over the batch's CSR with
 *    the core mask as filter (src/multi/runner_multi.cuh:715-729, 1062-1076), then for
 *    batches > 0 RAFT merge_labels into the accumulated labels
 *    (third_party/cuml/cpp/src/dbscan/mergelabels/runner.cuh:25-36, runner_multi.cuh:731-736).
 *    RAFT is not vendored in the reference; its published algorithm is restated literally:
 *      weak_cc: labels[i] = core ? i+1 : MAX over all N; then, until no core label changes,
 *        every batch row r visits its neighbours j: a core r lowers label[j] to label[r];
 *        any r adopts a smaller label of a core neighbour j.
 *      merge_labels: R[i] = i; until stable, for every core i with la = A[i]-1, lb = B[i]-1:
 *        if R[la] != R[lb], both are lowered to R[min(R[la], R[lb])]; then
 *        A[i] = min(map(A[i]), map(B[i])) with map(MAX) = MAX, map(v) = R[v-1]+1.
 *  - final relabel: RAFT make_monotonic with MAX filtered, then MAX -> -1, v -> v-1
 *    (src/multi/cuml_stages.cuh:196-218): cluster ids are the ranks of the distinct
 *    non-noise labels.
 *  - batch partition: rows [b*batch_size, min(N, (b+1)*batch_size)), batches in ascending
 *    order for labelling (src/multi/runner_multi.cuh:676-739).
 *
 * Parity pinning: tests/test_oracle_golden.py checks this file against the 13 golden label
 * bundles shipped with the reference (the *.labels.npz files under official-campaign-v1/.../validation) and
 * the reference's recorded selftest answers.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

#define DBMO_NO_NEIGHBOR 255
#define DBMO_MAX_EPS 16
#define DBMO_LABEL_MAX INT32_MAX

/* ------------------------------------------------------------------------------------ */
/* pair arithmetic                                                                       */
/* ------------------------------------------------------------------------------------ */

/* Code of a squared distance: smallest e with acc <= eps2[e]; eps2 is non-decreasing. */
static inline uint8_t code_of(float acc, const float* eps2, int k)
{
  if (!(acc <= eps2[k - 1])) return DBMO_NO_NEIGHBOR;
  for (int e = 0; e < k; ++e)
    if (acc <= eps2[e]) return (uint8_t)e;
  return DBMO_NO_NEIGHBOR;
}

void dbmo_square_eps(const float* eps, int k, float* eps2)
{
  for (int e = 0; e < k; ++e) {
    volatile float v = eps[e] * eps[e]; /* rounded to float, as the reference host does */
    eps2[e] = v;
  }
}

/* Candidate points transposed into blocks of 16 (xt[block][t][lane]) so that the CPU loop
 * runs 16 independent FMA chains side by side; no chain is ever reassociated. */
#define DBMO_LANES 16
static float* transpose_blocks(const float* x, int64_t n, int64_t d)
{
  const int64_t nblk = (n + DBMO_LANES - 1) / DBMO_LANES;
  float* xt = (float*)malloc(sizeof(float) * (size_t)nblk * (size_t)d * DBMO_LANES);
  if (!xt) return NULL;
  for (int64_t b = 0; b < nblk; ++b)
    for (int64_t t = 0; t < d; ++t)
      for (int64_t l = 0; l < DBMO_LANES; ++l) {
        const int64_t j = b * DBMO_LANES + l;
        xt[((size_t)b * (size_t)d + (size_t)t) * DBMO_LANES + (size_t)l] = j < n ? x[j * d + t] : 0.0f;
      }
  return xt;
}

static void row_block_codes_generic(const float* x, const float* xt, int64_t n, int64_t d, int64_t i,
                            const float* eps2, int k, uint8_t* out /* n */)
{
  const float* q = x + i * d;
  for (int64_t j0 = 0, b = 0; j0 < n; j0 += DBMO_LANES, ++b) {
    const int64_t cnt = (n - j0) < DBMO_LANES ? (n - j0) : DBMO_LANES;
    const float* blk = xt + (size_t)b * (size_t)d * DBMO_LANES;
    float acc[DBMO_LANES];
    for (int l = 0; l < DBMO_LANES; ++l) acc[l] = 0.0f;
    for (int64_t t = 0; t < d; ++t) {
      const float qt = q[t];
      const float* col = blk + t * DBMO_LANES;
#pragma GCC ivdep
      for (int l = 0; l < DBMO_LANES; ++l) {
        const float diff = qt - col[l];
        acc[l] = fmaf(diff, diff, acc[l]);
      }
    }
    for (int64_t l = 0; l < cnt; ++l) out[j0 + l] = code_of(acc[l], eps2, k);
  }
}

__attribute__((target("avx2,fma"))) static void row_block_codes_fma(const float* x, const float* xt, int64_t n, int64_t d, int64_t i,
                            const float* eps2, int k, uint8_t* out /* n */)
{
  const float* q = x + i * d;
  for (int64_t j0 = 0, b = 0; j0 < n; j0 += DBMO_LANES, ++b) {
    const int64_t cnt = (n - j0) < DBMO_LANES ? (n - j0) : DBMO_LANES;
    const float* blk = xt + (size_t)b * (size_t)d * DBMO_LANES;
    float acc[DBMO_LANES];
    for (int l = 0; l < DBMO_LANES; ++l) acc[l] = 0.0f;
    for (int64_t t = 0; t < d; ++t) {
      const float qt = q[t];
      const float* col = blk + t * DBMO_LANES;
#pragma GCC ivdep
      for (int l = 0; l < DBMO_LANES; ++l) {
        const float diff = qt - col[l];
        acc[l] = fmaf(diff, diff, acc[l]);
      }
    }
    for (int64_t l = 0; l < cnt; ++l) out[j0 + l] = code_of(acc[l], eps2, k);
  }
}

/* Hardware FMA when the host has it (fmaf is exact either way: the libm call and the
 * vfmadd instruction both round once). */
static void row_block_codes(const float* x, const float* xt, int64_t n, int64_t d, int64_t i,
                            const float* eps2, int k, uint8_t* out)
{
  static int have_fma = -1;
  if (have_fma < 0) {
    __builtin_cpu_init();
    have_fma = __builtin_cpu_supports("fma") && __builtin_cpu_supports("avx2");
  }
  if (have_fma)
    row_block_codes_fma(x, xt, n, d, i, eps2, k, out);
  else
    row_block_codes_generic(x, xt, n, d, i, eps2, k, out);
}

/* ------------------------------------------------------------------------------------ */
/* neighbourhood: codes, degrees, max-eps CSR                                           */
/* ------------------------------------------------------------------------------------ */

/* One row: codes into `out` (n bytes) and its k cumulative degrees. */
static void one_row(const float* x, const float* xt, int64_t n, int64_t d, int64_t i,
                    const float* eps2, int k, uint8_t* out, int32_t* deg, int64_t rows, int64_t r)
{
  row_block_codes(x, xt, n, d, i, eps2, k, out);
  int32_t hist[DBMO_MAX_EPS + 1];
  memset(hist, 0, sizeof(hist));
  for (int64_t j = 0; j < n; ++j) {
    const uint8_t c = out[j];
    hist[c == DBMO_NO_NEIGHBOR ? k : c] += 1;
  }
  int32_t run = 0;
  for (int e = 0; e < k; ++e) {
    run += hist[e];
    deg[(size_t)e * (size_t)rows + (size_t)r] = run;
  }
}

typedef struct {
  const float* x;
  const float* xt;
  int64_t n, d, row0, rows;
  const float* eps2;
  int k;
  int32_t* deg;
  uint8_t* codes;
  int64_t next; /* shared row cursor, taken with __atomic_fetch_add */
  int failed;
} rows_job_t;

static void* rows_worker(void* arg)
{
  rows_job_t* job = (rows_job_t*)arg;
  uint8_t* line = job->codes ? NULL : (uint8_t*)malloc((size_t)job->n);
  if (!job->codes && !line) {
    __atomic_store_n(&job->failed, 1, __ATOMIC_RELAXED);
    return NULL;
  }
  for (;;) {
    const int64_t r = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (r >= job->rows) break;
    uint8_t* out = job->codes ? job->codes + (size_t)r * (size_t)job->n : line;
    one_row(job->x, job->xt, job->n, job->d, job->row0 + r, job->eps2, job->k, out, job->deg,
            job->rows, r);
  }
  free(line);
  return NULL;
}

/* Number of host threads: `threads` if > 0, else every online CPU. */
int dbmo_default_threads(void)
{
  const long c = sysconf(_SC_NPROCESSORS_ONLN);
  return c > 0 ? (int)c : 1;
}

/*
 * Per-pair codes and per-eps degrees for rows [row0, row0+rows) against all n points.
 *   deg:   k x rows, deg[e*rows + r] = #{j : code(row0+r, j) <= e}
 *   codes: optional rows x n bytes (NULL to skip)
 * Rows are spread over `threads` pthreads (<= 0: every online CPU).  Returns 0, -1 on bad
 * arguments, -2 on allocation failure.
 */
int dbmo_codes_degrees(const float* x, int64_t n, int64_t d, const float* eps2, int k,
                       int64_t row0, int64_t rows, int32_t* deg, uint8_t* codes, int threads)
{
  if (k < 1 || k > DBMO_MAX_EPS || n < 1 || d < 1 || rows < 0) return -1;
  int t = threads > 0 ? threads : dbmo_default_threads();
  if (t > 256) t = 256;
  if ((int64_t)t > rows) t = rows > 0 ? (int)rows : 1;
  float* xt = transpose_blocks(x, n, d);
  if (!xt) return -2;
  rows_job_t job = {x, xt, n, d, row0, rows, eps2, k, deg, codes, 0, 0};
  pthread_t tid[256];
  int started = 0;
  for (int w = 1; w < t; ++w)
    if (pthread_create(&tid[started], NULL, rows_worker, &job) == 0) ++started;
  rows_worker(&job);
  for (int w = 0; w < started; ++w) pthread_join(tid[w], NULL);
  free(xt);
  return job.failed ? -2 : 0;
}

typedef struct {
  int64_t* off;  /* n+1 */
  int32_t* col;  /* nnz, ascending per row, self included */
  uint8_t* code; /* nnz */
} csr_t;

static void csr_free(csr_t* g)
{
  free(g->off);
  free(g->col);
  free(g->code);
}

/* Max-eps neighbour lists (with per-entry codes) and per-eps degrees for all n rows. */
static int build_graph(const float* x, int64_t n, int64_t d, const float* eps2, int k,
                       csr_t* g, int32_t* deg /* k*n */)
{
  const int64_t block = 256;
  uint8_t* codes = (uint8_t*)malloc((size_t)block * (size_t)n);
  int32_t* bdeg = (int32_t*)malloc(sizeof(int32_t) * (size_t)k * (size_t)block);
  g->off = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
  int64_t cap = n * 8 + 64, nnz = 0;
  g->col = (int32_t*)malloc(sizeof(int32_t) * (size_t)cap);
  g->code = (uint8_t*)malloc((size_t)cap);
  if (!codes || !bdeg || !g->off || !g->col || !g->code) return -2;
  for (int64_t r0 = 0; r0 < n; r0 += block) {
    const int64_t rows = (n - r0) < block ? (n - r0) : block;
    dbmo_codes_degrees(x, n, d, eps2, k, r0, rows, bdeg, codes, 0);
    for (int64_t r = 0; r < rows; ++r) {
      for (int e = 0; e < k; ++e)
        deg[(size_t)e * (size_t)n + (size_t)(r0 + r)] = bdeg[(size_t)e * (size_t)rows + (size_t)r];
      const uint8_t* line = codes + (size_t)r * (size_t)n;
      for (int64_t j = 0; j < n; ++j) {
        if (line[j] == DBMO_NO_NEIGHBOR) continue;
        if (nnz == cap) {
          cap *= 2;
          g->col = (int32_t*)realloc(g->col, sizeof(int32_t) * (size_t)cap);
          g->code = (uint8_t*)realloc(g->code, (size_t)cap);
          if (!g->col || !g->code) return -2;
        }
        g->col[nnz] = (int32_t)j;
        g->code[nnz] = line[j];
        ++nnz;
      }
      g->off[r0 + r + 1] = nnz;
    }
  }
  free(codes);
  free(bdeg);
  return 0;
}

/* ------------------------------------------------------------------------------------ */
/* labelling: literal restatement of RAFT weak_cc_batched + merge_labels                 */
/* ------------------------------------------------------------------------------------ */

static void weak_cc_batch(int32_t* lab, const csr_t* g, int e, const uint8_t* core,
                          int64_t n, int64_t start, int64_t rows)
{
  for (int64_t i = 0; i < n; ++i) lab[i] = core[i] ? (int32_t)(i + 1) : DBMO_LABEL_MAX;
  int changed = 1;
  while (changed) {
    changed = 0;
    for (int64_t r = start; r < start + rows; ++r) {
      int32_t ci = lab[r];
      int ci_mod = 0;
      const int r_core = core[r];
      for (int64_t p = g->off[r]; p < g->off[r + 1]; ++p) {
        if (g->code[p] > e) continue;
        const int32_t j = g->col[p];
        const int32_t cj = lab[j];
        if (ci < cj && r_core) {
          lab[j] = ci; /* atomicMin in RAFT; sequential here */
          if (core[j]) changed = 1;
        } else if (ci > cj && core[j]) {
          ci = cj;
          ci_mod = 1;
        }
      }
      if (ci_mod && ci < lab[r]) {
        lab[r] = ci;
        if (r_core) changed = 1;
      }
    }
  }
}

static void merge_labels(int32_t* a, const int32_t* b, const uint8_t* core, int32_t* R, int64_t n)
{
  for (int64_t i = 0; i < n; ++i) R[i] = (int32_t)i;
  int changed = 1;
  while (changed) {
    changed = 0;
    for (int64_t i = 0; i < n; ++i) {
      if (!core[i]) continue;
      const int32_t la = a[i] - 1, lb = b[i] - 1;
      const int32_t ra = R[la], rb = R[lb];
      if (ra != rb) {
        changed = 1;
        const int32_t rmin = R[ra < rb ? ra : rb];
        if (rmin < R[la]) R[la] = rmin;
        if (rmin < R[lb]) R[lb] = rmin;
      }
    }
  }
  for (int64_t i = 0; i < n; ++i) {
    const int32_t la = a[i], lb = b[i];
    const int32_t ra = (la == DBMO_LABEL_MAX) ? DBMO_LABEL_MAX : R[la - 1] + 1;
    const int32_t rb = (lb == DBMO_LABEL_MAX) ? DBMO_LABEL_MAX : R[lb - 1] + 1;
    a[i] = ra < rb ? ra : rb;
  }
}

static int cmp_i32(const void* p, const void* q)
{
  const int32_t a = *(const int32_t*)p, b = *(const int32_t*)q;
  return (a > b) - (a < b);
}

/* make_monotonic(filter MAX) followed by MAX -> -1, v -> v-1. */
static void relabel(int32_t* lab, int64_t n, int32_t* scratch)
{
  int64_t m = 0;
  for (int64_t i = 0; i < n; ++i)
    if (lab[i] != DBMO_LABEL_MAX) scratch[m++] = lab[i];
  qsort(scratch, (size_t)m, sizeof(int32_t), cmp_i32);
  int64_t u = 0;
  for (int64_t i = 0; i < m; ++i)
    if (u == 0 || scratch[u - 1] != scratch[i]) scratch[u++] = scratch[i];
  for (int64_t i = 0; i < n; ++i) {
    if (lab[i] == DBMO_LABEL_MAX) {
      lab[i] = -1;
      continue;
    }
    int64_t lo = 0, hi = u - 1;
    while (lo < hi) {
      const int64_t mid = (lo + hi) / 2;
      if (scratch[mid] < lab[i]) lo = mid + 1; else hi = mid;
    }
    lab[i] = (int32_t)lo;
  }
}

/*
 * Full grid fit.
 *   x: n x d row-major float32; eps[k] ascending unique; minpts[l] ascending unique.
 *   batch_size: rows per labelling batch (>= 1); the partition decides how ambiguous
 *     border points resolve, exactly as in the reference.
 *   labels: k*l*n int32 out, config = e*l + m, -1 noise.
 *   core_out: optional k*l*n bytes (1 = core).
 *   deg_out: optional k*n int32 per-eps degrees.
 * Returns 0, or a negative value on invalid arguments / allocation failure.
 */
int dbmo_fit_multi(const float* x, int64_t n, int64_t d, const float* eps, int k,
                   const int32_t* minpts, int l, int64_t batch_size, int32_t* labels,
                   uint8_t* core_out, int32_t* deg_out)
{
  if (n < 1 || d < 1 || k < 1 || k > DBMO_MAX_EPS || l < 1 || batch_size < 1) return -1;
  if (n >= (int64_t)INT32_MAX) return -1;
  float eps2[DBMO_MAX_EPS];
  dbmo_square_eps(eps, k, eps2);

  csr_t g = {0};
  int32_t* deg = (int32_t*)malloc(sizeof(int32_t) * (size_t)k * (size_t)n);
  uint8_t* core = (uint8_t*)malloc((size_t)n);
  int32_t* tmp = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  int32_t* R = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  if (!deg || !core || !tmp || !R) return -2;
  int rc = build_graph(x, n, d, eps2, k, &g, deg);
  if (rc != 0) return rc;
  if (deg_out) memcpy(deg_out, deg, sizeof(int32_t) * (size_t)k * (size_t)n);

  const int64_t nb = (n + batch_size - 1) / batch_size;
  for (int e = 0; e < k; ++e) {
    for (int m = 0; m < l; ++m) {
      const int64_t cfg = (int64_t)e * l + m;
      for (int64_t i = 0; i < n; ++i) core[i] = deg[(size_t)e * (size_t)n + (size_t)i] >= minpts[m];
      if (core_out) memcpy(core_out + (size_t)cfg * (size_t)n, core, (size_t)n);
      int32_t* out = labels + (size_t)cfg * (size_t)n;
      for (int64_t b = 0; b < nb; ++b) {
        const int64_t start = b * batch_size;
        const int64_t rows = (n - start) < batch_size ? (n - start) : batch_size;
        weak_cc_batch(b == 0 ? out : tmp, &g, e, core, n, start, rows);
        if (b > 0) merge_labels(out, tmp, core, R, n);
      }
      relabel(out, n, tmp);
    }
  }
  csr_free(&g);
  free(deg);
  free(core);
  free(tmp);
  free(R);
  return 0;
}

/* Route rule of the reference's cuVS backend (runner_multi.cuh:405-415, constants :368,380):
 * annotate iff nnz*D*40 < (k-1)*(pairs*D + 6e10), evaluated in long double. */
int dbmo_annotate_pays(int64_t nnz, int64_t pairs, int k, int64_t d)
{
  const long double cost_annotate = (long double)nnz * (long double)d * 40.0L;
  const long double cost_searches =
    (long double)(k - 1) * ((long double)pairs * (long double)d + 60000000000.0L);
  return cost_annotate < cost_searches;
}

/* ------------------------------------------------------------------------------------ */
/* streaming fit: the same results as dbmo_fit_multi, memory bounded by one row batch     */
/* ------------------------------------------------------------------------------------ */
/*
 * dbmo_fit_multi_stream computes exactly what dbmo_fit_multi computes (same codes, degrees,
 * labels) with the reference's own pass structure (runner_multi.cuh:624-739): a first pass over
 * all rows for the per-eps degrees, then per row batch the batch's neighbour lists (rows of the
 * batch x all points, rebuilt from the distances, as the reference's pass 2 rebuilds each
 * batch's CSR), labelled and merged for every configuration before the next batch.  Only one
 * batch's lists are held at a time.  Two changes make it fast enough for the full-size
 * configurations, neither of which changes a result:
 *   - four query rows share one read of each 16-point candidate block;
 *   - after every 8 dims, a block whose 4 x 16 partial sums all exceed the largest eps^2 is
 *     dropped: fma(diff, diff, acc) >= acc, so those pairs end above the cutoff anyway (the
 *     reference's generic kernel breaks the same way per pair, eps_neighborhood.cuh:247).
 * Configurations are labelled in parallel (each has its own label, scratch and merge arrays;
 * the weak-CC and merge of one configuration stay sequential and literal).
 */
#define DBMO_QROWS 4

typedef struct {
  int32_t hist[DBMO_QROWS][DBMO_MAX_EPS + 1];
  int32_t* col[DBMO_QROWS];  /* NULL: counts only */
  uint8_t* code[DBMO_QROWS];
  int64_t fill[DBMO_QROWS];
} scan_out_t;

static inline __attribute__((always_inline)) void scan_rows_body(const float* x, const float* xt, int64_t n,
                                                                 int64_t d, const int64_t* qi, int nr,
                                                                 const float* eps2, int k, scan_out_t* o)
{
  const float cutoff = eps2[k - 1];
  const float* qp[DBMO_QROWS];
  for (int r = 0; r < DBMO_QROWS; ++r) qp[r] = x + qi[r < nr ? r : (nr > 1 ? nr - 1 : 0)] * d;
  for (int64_t j0 = 0, b = 0; j0 < n; j0 += DBMO_LANES, ++b) {
    const float* blk = xt + (size_t)b * (size_t)d * DBMO_LANES;
    float acc[DBMO_QROWS][DBMO_LANES];
    for (int r = 0; r < DBMO_QROWS; ++r)
      for (int l = 0; l < DBMO_LANES; ++l) acc[r][l] = 0.0f;
    int alive = 1;
    int64_t t = 0;
    while (t < d) {
      const int64_t te = (t + 8 < d) ? t + 8 : d;
      for (; t < te; ++t) {
        const float* col = blk + t * DBMO_LANES;
        for (int r = 0; r < DBMO_QROWS; ++r) {
          const float qt = qp[r][t];
#pragma GCC ivdep
          for (int l = 0; l < DBMO_LANES; ++l) {
            const float diff = qt - col[l];
            acc[r][l] = fmaf(diff, diff, acc[r][l]);
          }
        }
      }
      if (t < d) {
        int any = 0;
        for (int r = 0; r < DBMO_QROWS; ++r)
          for (int l = 0; l < DBMO_LANES; ++l) any |= acc[r][l] <= cutoff;
        if (!any) {
          alive = 0;
          break;
        }
      }
    }
    if (!alive) continue;
    const int64_t cnt = (n - j0) < DBMO_LANES ? (n - j0) : DBMO_LANES;
    for (int r = 0; r < nr; ++r) {
      for (int64_t l = 0; l < cnt; ++l) {
        const uint8_t c = code_of(acc[r][l], eps2, k);
        if (c == DBMO_NO_NEIGHBOR) continue;
        o->hist[r][c] += 1;
        if (o->col[r]) {
          o->col[r][o->fill[r]] = (int32_t)(j0 + l);
          o->code[r][o->fill[r]] = c;
          o->fill[r] += 1;
        }
      }
    }
  }
}

__attribute__((target("avx2,fma"))) static void scan_rows_fma(const float* x, const float* xt, int64_t n, int64_t d,
                                                              const int64_t* qi, int nr, const float* eps2, int k,
                                                              scan_out_t* o)
{
  scan_rows_body(x, xt, n, d, qi, nr, eps2, k, o);
}

static void scan_rows_generic(const float* x, const float* xt, int64_t n, int64_t d, const int64_t* qi, int nr,
                              const float* eps2, int k, scan_out_t* o)
{
  scan_rows_body(x, xt, n, d, qi, nr, eps2, k, o);
}

static void scan_rows(const float* x, const float* xt, int64_t n, int64_t d, const int64_t* qi, int nr,
                      const float* eps2, int k, scan_out_t* o)
{
  static int have_fma = -1;
  if (have_fma < 0) {
    __builtin_cpu_init();
    have_fma = __builtin_cpu_supports("fma") && __builtin_cpu_supports("avx2");
  }
  if (have_fma)
    scan_rows_fma(x, xt, n, d, qi, nr, eps2, k, o);
  else
    scan_rows_generic(x, xt, n, d, qi, nr, eps2, k, o);
}

typedef struct {
  const float* x;
  const float* xt;
  int64_t n, d;
  const float* eps2;
  int k;
  int64_t row0, rows;     /* rows [row0, row0 + rows) */
  int32_t* deg;           /* pass 1: k x n cumulative degrees (NULL in pass 2) */
  const int64_t* off;     /* pass 2: rows + 1 list offsets (relative to the batch) */
  int32_t* col;           /* pass 2: neighbour lists */
  uint8_t* code;
  int64_t next;           /* shared cursor over groups of DBMO_QROWS rows */
} stream_job_t;

static void* stream_worker(void* arg)
{
  stream_job_t* job = (stream_job_t*)arg;
  const int64_t groups = (job->rows + DBMO_QROWS - 1) / DBMO_QROWS;
  for (;;) {
    const int64_t g = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (g >= groups) break;
    int64_t qi[DBMO_QROWS];
    int nr = 0;
    for (int r = 0; r < DBMO_QROWS; ++r) {
      const int64_t rr = g * DBMO_QROWS + r;
      if (rr < job->rows) qi[nr++] = job->row0 + rr;
    }
    scan_out_t o;
    memset(&o, 0, sizeof(o));
    if (job->col) {
      for (int r = 0; r < nr; ++r) {
        const int64_t lr = qi[r] - job->row0;
        o.col[r] = job->col + job->off[lr];
        o.code[r] = job->code + job->off[lr];
      }
    }
    scan_rows(job->x, job->xt, job->n, job->d, qi, nr, job->eps2, job->k, &o);
    if (job->deg) {
      for (int r = 0; r < nr; ++r) {
        int32_t run = 0;
        for (int e = 0; e < job->k; ++e) {
          run += o.hist[r][e];
          job->deg[(size_t)e * (size_t)job->n + (size_t)qi[r]] = run;
        }
      }
    }
  }
  return NULL;
}

static void run_stream_job(stream_job_t* job, int threads)
{
  pthread_t tid[256];
  int started = 0;
  for (int w = 1; w < threads; ++w)
    if (pthread_create(&tid[started], NULL, stream_worker, job) == 0) ++started;
  stream_worker(job);
  for (int w = 0; w < started; ++w) pthread_join(tid[w], NULL);
}

/* weak_cc_batch over the batch-local lists (row r of the batch at off[r - start]). */
static void weak_cc_batch_local(int32_t* lab, const int64_t* off, const int32_t* col, const uint8_t* code, int e,
                                const uint8_t* core, int64_t n, int64_t start, int64_t rows)
{
  for (int64_t i = 0; i < n; ++i) lab[i] = core[i] ? (int32_t)(i + 1) : DBMO_LABEL_MAX;
  int changed = 1;
  while (changed) {
    changed = 0;
    for (int64_t r = start; r < start + rows; ++r) {
      int32_t ci = lab[r];
      int ci_mod = 0;
      const int r_core = core[r];
      for (int64_t p = off[r - start]; p < off[r - start + 1]; ++p) {
        if (code[p] > e) continue;
        const int32_t j = col[p];
        const int32_t cj = lab[j];
        if (ci < cj && r_core) {
          lab[j] = ci;
          if (core[j]) changed = 1;
        } else if (ci > cj && core[j]) {
          ci = cj;
          ci_mod = 1;
        }
      }
      if (ci_mod && ci < lab[r]) {
        lab[r] = ci;
        if (r_core) changed = 1;
      }
    }
  }
}

typedef struct {
  int64_t n, start, rows, batch;
  int k, l;
  const int32_t* deg;
  const int32_t* minpts;
  const int64_t* off;
  const int32_t* col;
  const uint8_t* code;
  int32_t* labels;   /* k*l x n */
  int32_t* tmp;      /* k*l x n scratch */
  int32_t* R;        /* k*l x n merge map */
  uint8_t* core;     /* k*l x n */
  int64_t next;
} label_job_t;

static void* label_worker(void* arg)
{
  label_job_t* job = (label_job_t*)arg;
  const int64_t C = (int64_t)job->k * job->l;
  for (;;) {
    const int64_t cfg = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (cfg >= C) break;
    const int e = (int)(cfg / job->l);
    const size_t base = (size_t)cfg * (size_t)job->n;
    int32_t* out = job->labels + base;
    weak_cc_batch_local(job->batch == 0 ? out : job->tmp + base, job->off, job->col, job->code, e, job->core + base,
                        job->n, job->start, job->rows);
    if (job->batch > 0) merge_labels(out, job->tmp + base, job->core + base, job->R + base, job->n);
  }
  return NULL;
}

static void* relabel_worker(void* arg)
{
  label_job_t* job = (label_job_t*)arg;
  const int64_t C = (int64_t)job->k * job->l;
  for (;;) {
    const int64_t cfg = __atomic_fetch_add(&job->next, 1, __ATOMIC_RELAXED);
    if (cfg >= C) break;
    const size_t base = (size_t)cfg * (size_t)job->n;
    relabel(job->labels + base, job->n, job->tmp + base);
  }
  return NULL;
}

static void run_label_job(label_job_t* job, int threads, void* (*fn)(void*))
{
  pthread_t tid[256];
  int started = 0;
  job->next = 0;
  for (int w = 1; w < threads; ++w)
    if (pthread_create(&tid[started], NULL, fn, job) == 0) ++started;
  fn(job);
  for (int w = 0; w < started; ++w) pthread_join(tid[w], NULL);
}

/*
 * Same contract as dbmo_fit_multi, plus `threads` (<= 0: every online CPU) and an optional
 * `nnz_out` (sum over batches of the max-eps list entries, self pairs included).
 */
int dbmo_fit_multi_stream(const float* x, int64_t n, int64_t d, const float* eps, int k, const int32_t* minpts,
                          int l, int64_t batch_size, int32_t* labels, uint8_t* core_out, int32_t* deg_out,
                          int threads, int64_t* nnz_out)
{
  if (n < 1 || d < 1 || k < 1 || k > DBMO_MAX_EPS || l < 1 || batch_size < 1) return -1;
  if (n >= (int64_t)INT32_MAX) return -1;
  int t = threads > 0 ? threads : dbmo_default_threads();
  if (t > 256) t = 256;
  float eps2[DBMO_MAX_EPS];
  dbmo_square_eps(eps, k, eps2);
  const int64_t C = (int64_t)k * l;
  float* xt = transpose_blocks(x, n, d);
  int32_t* deg = (int32_t*)malloc(sizeof(int32_t) * (size_t)k * (size_t)n);
  int32_t* tmp = (int32_t*)malloc(sizeof(int32_t) * (size_t)C * (size_t)n);
  int32_t* R = (int32_t*)malloc(sizeof(int32_t) * (size_t)C * (size_t)n);
  uint8_t* core = (uint8_t*)malloc((size_t)C * (size_t)n);
  int64_t* off = (int64_t*)malloc(sizeof(int64_t) * ((size_t)(batch_size < n ? batch_size : n) + 1));
  if (!xt || !deg || !tmp || !R || !core || !off) return -2;

  /* pass 1: per-eps degrees of every row */
  stream_job_t job;
  memset(&job, 0, sizeof(job));
  job.x = x;
  job.xt = xt;
  job.n = n;
  job.d = d;
  job.eps2 = eps2;
  job.k = k;
  job.row0 = 0;
  job.rows = n;
  job.deg = deg;
  run_stream_job(&job, t);
  if (deg_out) memcpy(deg_out, deg, sizeof(int32_t) * (size_t)k * (size_t)n);
  for (int e = 0; e < k; ++e)
    for (int m = 0; m < l; ++m) {
      uint8_t* c = core + ((size_t)e * l + m) * (size_t)n;
      for (int64_t i = 0; i < n; ++i) c[i] = deg[(size_t)e * (size_t)n + (size_t)i] >= minpts[m];
    }
  if (core_out) memcpy(core_out, core, (size_t)C * (size_t)n);

  /* pass 2: per batch, its neighbour lists, then every configuration's weak-CC + merge */
  const int64_t nb = (n + batch_size - 1) / batch_size;
  int64_t nnz_total = 0;
  for (int64_t b = 0; b < nb; ++b) {
    const int64_t start = b * batch_size;
    const int64_t rows = (n - start) < batch_size ? (n - start) : batch_size;
    off[0] = 0;
    for (int64_t r = 0; r < rows; ++r) off[r + 1] = off[r] + deg[(size_t)(k - 1) * (size_t)n + (size_t)(start + r)];
    const int64_t nnz = off[rows];
    nnz_total += nnz;
    int32_t* col = (int32_t*)malloc(sizeof(int32_t) * (size_t)(nnz > 0 ? nnz : 1));
    uint8_t* code = (uint8_t*)malloc((size_t)(nnz > 0 ? nnz : 1));
    if (!col || !code) return -2;
    memset(&job, 0, sizeof(job));
    job.x = x;
    job.xt = xt;
    job.n = n;
    job.d = d;
    job.eps2 = eps2;
    job.k = k;
    job.row0 = start;
    job.rows = rows;
    job.off = off;
    job.col = col;
    job.code = code;
    run_stream_job(&job, t);
    label_job_t lj;
    memset(&lj, 0, sizeof(lj));
    lj.n = n;
    lj.start = start;
    lj.rows = rows;
    lj.batch = b;
    lj.k = k;
    lj.l = l;
    lj.deg = deg;
    lj.minpts = minpts;
    lj.off = off;
    lj.col = col;
    lj.code = code;
    lj.labels = labels;
    lj.tmp = tmp;
    lj.R = R;
    lj.core = core;
    run_label_job(&lj, t, label_worker);
    free(col);
    free(code);
  }
  label_job_t rj;
  memset(&rj, 0, sizeof(rj));
  rj.n = n;
  rj.k = k;
  rj.l = l;
  rj.labels = labels;
  rj.tmp = tmp;
  run_label_job(&rj, t, relabel_worker);
  if (nnz_out) *nnz_out = nnz_total;
  free(xt);
  free(deg);
  free(tmp);
  free(R);
  free(core);
  free(off);
  return 0;
}

/* The reference's per-pair value acc (eps_neighborhood.cuh:151-158: sequential fma over the
 * dims) for m pairs (a[i*d ..], b[i*d ..]) -> out[i]; used by tests to plant pairs exactly at
 * an eps boundary. */
void dbmo_pair_chain(const float* a, const float* b, int64_t m, int64_t d, float* out)
{
  for (int64_t i = 0; i < m; ++i) {
    float acc = 0.0f;
    for (int64_t t = 0; t < d; ++t) {
      const float diff = a[i * d + t] - b[i * d + t];
      acc = fmaf(diff, diff, acc);
    }
    out[i] = acc;
  }
}
