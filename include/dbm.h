/*
 * dbm.h -- C ABI of the B200-native multi-parameter DBSCAN (`fit_multi`) library, libdbm.so.
 *
 * One call clusters N points under every (eps, minPts) pair of a k x l grid and returns k*l
 * label vectors (config = e*l + m, eps-major, -1 = noise) plus the k*l core masks.  Labels
 * are identical, bit for bit, to the reference implementation's for the same float32 input
 * and the same batch partition.
 *
 * Reference interfaces replaced (Math-BUG/cuML-DBSCANMulti):
 *   dbm_fit_multi          ML::Dbscan::Multi::fit_multi<float, Index_>
 *                          (src/multi/runner_multi.cuh:1290-1307), as driven by
 *                          fit_com_handle (src/main.cu:498-598)
 *   dbm_fit_multi_host     the CLI's fit() path with host buffers: H2D of points, fit,
 *                          D2H of labels with the range check (src/main.cu:527-598)
 *   dbm_neighbor_counts    VertexDeg::run_multi's per-eps degrees
 *                          (src/multi/eps_neighborhood.cuh:440-479)
 *   dbm_batch_size         compute_batch_size_multi (src/multi/runner_multi.cuh:458-499)
 *   dbm_max_bytes_for_batch_size  max_bytes_for_batch_size (runner_multi.cuh:437-447)
 *   dbm_annotate_pays      anotar_compensa (runner_multi.cuh:405-415)
 *   dbm_options.route      rota_forcada (runner_multi.cuh:426-430)
 *   dbm_options.csr_cap_bytes  csr_teto_de_teste (runner_multi.cuh:145-149)
 *   dbm_stats              ExecutionStats / last_execution_stats (runner_multi.cuh:175-208),
 *                          returned per call instead of thread-local
 *   dbm_handle             the caller-owned workspace + BuffersCsr pair reused across calls
 *                          (runner_multi.cuh:516-526, src/main.cu:621-645)
 *   dbm_build_info_json    write_build_json (src/main.cu:130-156)
 *
 * Conventions: every entry point returns DBM_OK (0) or a negative DBM_ERR_* code and never
 * aborts the process; a human-readable message goes to `err` (NUL-terminated, truncated
 * to err_len) when err != NULL.  Device pointers are plain CUDA device addresses on the
 * handle's device; `stream` is a cudaStream_t (NULL = the handle's own stream).  One fit
 * per handle at a time.
 */
#ifndef DBM_H
#define DBM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define DBM_OK 0
#define DBM_ERR_INVALID (-1)          /* bad argument: k outside 1..16 (eps_neighborhood.cuh:455),
                                         unsorted/duplicate lists, non-positive minPts, N<1 ... */
#define DBM_ERR_FIXED_BUFFERS (-2)    /* fixed buffers exceed the budget (runner_multi.cuh:474-479) */
#define DBM_ERR_INDEX_OVERFLOW (-3)   /* N too large for the index type (runner_multi.cuh:485-495) */
#define DBM_ERR_CSR_NOT_FIT (-4)      /* CSR does not fit after the batch corrections
                                         (runner_multi.cuh:1438-1445, 1456) */
#define DBM_ERR_CUDA (-5)             /* a CUDA runtime call failed */
#define DBM_ERR_OOM (-6)              /* device allocation failed */
#define DBM_ERR_NOT_CONVERGED (-7)    /* a bounded device wait or iteration limit ran out */
#define DBM_ERR_NO_DEVICE (-8)        /* no usable sm_100 device */
#define DBM_ERR_TOO_LARGE (-9)        /* N >= 2^28 (column index + code share one 32-bit word) */
#define DBM_ERR_NONFINITE (-10)       /* NaN/Inf in the points (src/main.cu:1419-1423) */

#define DBM_MAX_EPS 16

/* ---- options / statistics ------------------------------------------------------------ */
#define DBM_BACKEND_CUVS 0   /* batch sizing + per-batch route policy of the reference's
                                default (cuVS) backend */
#define DBM_BACKEND_CODES 1  /* batch sizing of the reference's codes backend; no routes */

#define DBM_ROUTE_AUTO 0
#define DBM_ROUTE_ANNOTATED 1
#define DBM_ROUTE_DENSE 2

/* values written to batch_routes[] */
#define DBM_BATCH_NOT_APPLICABLE 0
#define DBM_BATCH_ANNOTATED 1
#define DBM_BATCH_DENSE 2

typedef struct dbm_options {
  int backend;                /* DBM_BACKEND_* (reference CLI --backend; default cuvs) */
  int index_bits;             /* 0 = auto (64 iff N*N >= INT32_MAX), 32 or 64 (--index) */
  int route;                  /* DBM_ROUTE_* (--route) */
  int64_t neigh_per_row;      /* expected neighbours per row for batch sizing; 0 = N (--neigh-per-row) */
  uint64_t max_bytes_per_batch; /* memory budget; 0 = 80% of free + reusable (--max-mbytes-per-batch) */
  uint64_t csr_cap_bytes;     /* test knob: pretend only this much memory is free for the CSR
                                 check; 0 = real free memory */
} dbm_options;

typedef struct dbm_stats {
  uint64_t max_bytes_per_batch; /* effective budget */
  uint64_t batch_size;
  int32_t batches;
  int32_t attempts;
  int32_t batch_corrections;
  int32_t dense_batches;
  int32_t annotated_batches;
  int32_t index_bits;           /* index type the batch arithmetic used */
  int64_t max_nnz;              /* largest per-batch CSR (max eps, reference accounting) */
  int64_t total_nnz_max_eps;    /* sum over batches of the max-eps nnz (self pairs included) */
  int64_t unique_pairs;         /* distinct pairs i<j evaluated by the distance kernel */
  int64_t edges;                /* distinct neighbour pairs i<j within the largest eps */
  int32_t distance_passes;      /* 1, or 2 when the edge buffer had to grow */
  int32_t launches;             /* kernels this library launched during the call */
  double ms_distance;           /* device time of the distance kernel(s), if timing enabled */
  double ms_graph;              /* degrees, masks, CSR build */
  double ms_label;              /* per-batch compaction, connected components, merge */
  double ms_relabel;            /* final relabel */
  double dist_work_fraction;    /* fraction of all pair-dims (this shard's share of the tile
                                   pairs x D) the distance kernel computed: pruned tile pairs
                                   and warps whose pairs all exceed the largest eps stop early */
  double tile_pairs_kept;       /* fraction of tile pairs that survived the bounding-box bound */
  int64_t screened_tile_pairs;  /* tile pairs bounded by the tensor-core screen */
  int64_t fallback_tile_pairs;  /* of those and the unscreenable ones, handed to the exact tile kernel */
  int64_t screen_candidates;    /* pairs the screen could not exclude (each re-evaluated exactly) */
  double ms_screen;             /* device time of the screened-pass kernel alone, if timing enabled */
  int32_t streamed;             /* 1: the graph was built one row batch at a time (memory-bounded) */
  int32_t reserved0;
  uint64_t workspace_bytes;     /* the handle's device workspace after the call */
  int64_t nnz_per_eps[DBM_MAX_EPS]; /* directed neighbour entries per eps, self pairs excluded
                                       (sum over all rows of the reference's vd[e] minus N) */
} dbm_stats;

typedef struct dbm_handle dbm_handle;

/* ---- lifecycle ---------------------------------------------------------------------- */
/* Creates a handle on `device` (a CUDA ordinal).  `stream` may be NULL (the handle creates
 * its own non-blocking stream).  Returns NULL on failure (message in err). */
dbm_handle* dbm_create(int device, void* stream, char* err, size_t err_len);
/* Frees the handle's workspace and stream (if it owns it). */
void dbm_destroy(dbm_handle* h);
/* Bytes currently held by the handle's persistent workspace. */
uint64_t dbm_workspace_bytes(const dbm_handle* h);
/* Record per-phase device times into dbm_stats.ms_* (adds stream syncs; off by default). */
void dbm_set_phase_timing(dbm_handle* h, int enabled);

/* Distance pass selection (no counterpart in the reference, whose only path is the exact
 * per-pair search).  AUTO: the tensor-core screen bounds every surviving tile pair and the
 * exact fp32 chain re-evaluates each candidate, whenever N >= 4096, D <= 64 and
 * eps_max^2 >= 1e-20; otherwise the exact tile kernel.  EXACT: exact tile kernel only.
 * SCREENED: require the screen (DBM_ERR_INVALID when it does not apply).  Results are
 * identical in all modes. */
#define DBM_DISTANCE_AUTO 0
#define DBM_DISTANCE_EXACT 1
#define DBM_DISTANCE_SCREENED 2
int dbm_set_distance_mode(dbm_handle* h, int mode);

/* How the neighbour graph is held (the reference always rebuilds it per row batch, bounded by
 * its memory budget, runner_multi.cuh:1020-1041, 1100-1226).  AUTO: one pass writes every
 * neighbour pair and the whole max-eps CSR is built at once (24 bytes per neighbour pair) when
 * that, with the per-batch slabs, fits both the budget (dbm_options.max_bytes_per_batch, or its
 * automatic value) and the free device memory; otherwise the fit is memory-bounded: the degrees
 * come from the first pass, then each row batch's pairs are re-derived by a distance pass over the
 * tile pairs touching that batch and its rows of the CSR built into buffers sized by the largest
 * batch.  ONESHOT / STREAMED force one or the other (tests).  Labels are identical in every mode;
 * dbm_stats.streamed reports which ran.  dbm_distance_shard / dbm_fit_multi_from_graph always
 * hold the whole graph. */
#define DBM_GRAPH_AUTO 0
#define DBM_GRAPH_ONESHOT 1
#define DBM_GRAPH_STREAMED 2
int dbm_set_graph_mode(dbm_handle* h, int mode);

/* Test knob (fault injection without a GPU fault, like the reference's thread-local test knobs
 * csr_teto_de_teste / rota_forcada, runner_multi.cuh:145-160, 426-430): the retry bound of every
 * union-find hook in the labelling kernels (default 2^20, the largest accepted).  0 makes every
 * hook that is not already a no-op give up at once, so the fit returns DBM_ERR_NOT_CONVERGED
 * ("union-find retry bound ran out") and the handle stays usable.  DBM_ERR_INVALID for limit < 0. */
int dbm_set_union_retry_limit(dbm_handle* h, int limit);

/* ---- the fit ------------------------------------------------------------------------ */
/*
 * x_dev:        n x d float32, row-major, device
 * eps_host:     k values, strictly ascending, finite, > 0, <= sqrt(FLT_MAX); 1 <= k <= 16
 * min_pts_host: l values, strictly ascending, > 0
 * labels_dev:   k*l*n int32 out (device), config = e*l + m
 * core_dev:     optional k*l*n uint8 out (device), 1 = core point; NULL to skip
 * opt:          NULL = defaults (cuvs backend, auto index, auto route, worst-case
 *               neighbours, automatic budget)
 * stats:        optional out
 * batch_routes: optional out, DBM_BATCH_* per batch (ascending), at most routes_len entries;
 *               only the first stats->batches entries are written
 * Synchronises `stream` before returning (like the reference, which reads per-batch
 * sizes back to the host).
 */
int dbm_fit_multi(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host,
                  int k, const int32_t* min_pts_host, int l, int32_t* labels_dev, uint8_t* core_dev,
                  const dbm_options* opt, dbm_stats* stats, uint8_t* batch_routes, int routes_len,
                  void* stream, char* err, size_t err_len);

/* Same, with host buffers: copies x to the device, fits, copies labels (and optionally core
 * masks) back and checks -1 <= label < n.  x_host may be pageable or pinned. */
int dbm_fit_multi_host(dbm_handle* h, const float* x_host, int64_t n, int64_t d,
                       const float* eps_host, int k, const int32_t* min_pts_host, int l,
                       int32_t* labels_host, uint8_t* core_host, const dbm_options* opt,
                       dbm_stats* stats, uint8_t* batch_routes, int routes_len, char* err,
                       size_t err_len);

/* ---- multi-GPU stages (one process per GPU; the caller runs the collectives) ------------
 * dbm_fit_multi = dbm_distance_shard(shard 0 of 1) + dbm_fit_multi_from_graph(all configs).
 * With G ranks: rank r runs dbm_distance_shard(r, G); the hist arrays are summed across ranks
 * (all-reduce) and the neighbour pairs concatenated (all-gather, any order); every rank then
 * runs dbm_fit_multi_from_graph for its range of configs with the same options (an explicit
 * budget and csr_cap_bytes agreed across ranks keep the batch plan identical). */

/* Distance pass over the shard-th of nshards shares of the 128x128 tile pairs (i <= j): runs of
 * 64 consecutive work items (surviving tile pairs, or all tile pairs below 4096 points) dealt
 * round-robin over the shards, so the shares cost alike.
 * hist_dev: k*n int32 (zeroed here): pairs (i, j != i) of this shard per row and exact code.
 * edges_dev: edge_cap 64-bit words, i << 32 | code << 28 | j, one per neighbour pair i < j within
 * the largest eps found in this shard.  *edges_found receives the count; when it exceeds
 * edge_cap nothing is copied and the call must be repeated with a larger buffer.
 * Replaces the reference's pass-1 search over a row batch (runner_multi.cuh:627-655). */
int dbm_distance_shard(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host,
                       int k, int shard, int nshards, int32_t* hist_dev, uint64_t* edges_dev,
                       uint64_t edge_cap, uint64_t* edges_found, dbm_stats* stats /* optional: the
                       distance-pass fields (timers, screen and pruning counts) */, void* stream,
                       char* err, size_t err_len);

/* The exact tile-pair prune, sharded by work units (multi-GPU).  The prune's bound pass tests
 * every 128 x 128 tile pair (30.5M on 1M points); each rank tests a share of the
 * dbm_prune_units(n) units and the ranks all-gather the per-unit counts (int32 each) and keep masks
 * (dbm_prune_mask_words() uint32 words each), instead of every rank testing all of them.
 * dbm_prune_units: the number of units for n points (0 when n < 4096: no ordering and no prune
 * then, use dbm_distance_shard).
 * dbm_distance_prune_units: orders the points, builds XT and the tile boxes in the handle, and
 * writes the counts and masks of the units [unit_begin, unit_end) at their unit positions of
 * counts_dev / masks_dev (full-size arrays).  Asynchronous on `stream`.
 * dbm_distance_shard_pruned: dbm_distance_shard on the same handle and points, with the complete
 * counts and masks (gathered from every rank) in place of its own bound pass. */
int64_t dbm_prune_units(int64_t n);
int dbm_prune_mask_words(void);
int dbm_distance_prune_units(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host, int k,
                             int64_t unit_begin, int64_t unit_end, int32_t* counts_dev, uint32_t* masks_dev,
                             void* stream, char* err, size_t err_len);
int dbm_distance_shard_pruned(dbm_handle* h, const float* x_dev, int64_t n, int64_t d, const float* eps_host, int k,
                              int shard, int nshards, const int32_t* counts_dev, const uint32_t* masks_dev,
                              int32_t* hist_dev, uint64_t* edges_dev, uint64_t edge_cap, uint64_t* edges_found,
                              dbm_stats* stats, void* stream, char* err, size_t err_len);

/* Everything after the distance pass, from the complete per-code histograms (summed over all
 * shards) and the complete list of neighbour pairs: degrees, core masks, CSR, batch plan and
 * the labels of the configs [cfg_begin, cfg_end) (labels_dev rows outside the range are not
 * written).  Replaces runner_multi.cuh:657-746 (CSR, weak CC, merge, relabel). */
int dbm_fit_multi_from_graph(dbm_handle* h, int64_t n, int64_t d, const float* eps_host, int k,
                             const int32_t* min_pts_host, int l, const int32_t* hist_dev,
                             const uint64_t* edges_dev, uint64_t m_edges, int cfg_begin, int cfg_end,
                             int32_t* labels_dev, uint8_t* core_dev, const dbm_options* opt,
                             dbm_stats* stats, uint8_t* batch_routes, int routes_len, void* stream,
                             char* err, size_t err_len);

/* sklearn-style core sample indices of every labelling: out_dev[c*n + 0 ..] = the indices of
 * the core points of configuration c in ascending order, then -1 up to n (int32, device).
 * core_dev is the (configs x n) byte core mask of dbm_fit_multi.  This is the output cuML's
 * DBSCAN computes after its final relabel (third_party/cuml/cpp/src/dbscan/runner.cuh:406-430:
 * fill with -1, copy_if of the index range with the core mask as stencil), which the
 * reference's fit_multi does not expose. */
int dbm_core_sample_indices(dbm_handle* h, const uint8_t* core_dev, int64_t n, int configs, int32_t* out_dev,
                            void* stream, char* err, size_t err_len);

/* Per-eps neighbourhood sizes only (the point itself included): deg_dev[e*n + i] = #{j :
 * dist2(i, j) <= eps_e^2}, int32, device.  This is the degree vector the reference's
 * VertexDeg::run_multi produces per batch (src/multi/eps_neighborhood.cuh:440-479, vd[e]). */
int dbm_neighbor_counts(dbm_handle* h, const float* x_dev, int64_t n, int64_t d,
                        const float* eps_host, int k, int32_t* deg_dev, void* stream, char* err,
                        size_t err_len);

/* Allocation-free per-eps neighbourhood sizes.  No counterpart in the reference: it exists for
 * callers that cannot call cudaMalloc -- code under an allocator that owns all of the device's
 * memory (a framework's caching allocator, a hard per-process budget), or latency-critical code
 * that cannot take the device-wide synchronisation cudaMalloc/cudaFree imply.  Same output as
 * dbm_neighbor_counts (deg_dev[e*n + i], int32, device), but every byte of scratch comes from
 * one file-scope device array of 32 MiB (the padded dim-major copy of the points, 4*Dp*Npad
 * bytes with Dp = d rounded up to 4 and Npad = n rounded up to 4, plus 4*k*n bytes of counts and
 * 768 bytes of counters); larger inputs are rejected with DBM_ERR_TOO_LARGE.  The array is
 * resident on every GPU that uses the library until the process exits.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that device current.
 * Calls share the array, so calls that overlap on the GPU race; each call clears the parts that
 * must start at zero.  Cost: the exact tile kernel over every 128 x 128 tile pair, O(N^2 D),
 * without the spatial order, pruning or tensor-core screen of dbm_neighbor_counts (which needs
 * allocated buffers for them), so it can be orders of magnitude slower on large sparse inputs.
 * The call synchronises `stream` and reads a status word back to the host before it returns.
 * No handle is needed; stream NULL = the legacy default stream. */
int dbm_neighbor_counts_noalloc(const float* x_dev, int64_t n, int64_t d, const float* eps_host,
                                int k, int32_t* deg_dev, void* stream, char* err, size_t err_len);

/* ---- host-side rules (no device work) ---------------------------------------------- */
/* Batch rows for a budget; returns DBM_OK or DBM_ERR_FIXED_BUFFERS / DBM_ERR_INDEX_OVERFLOW. */
int dbm_batch_size(int64_t n, int k, int l, uint64_t max_bytes, int backend, int64_t neigh_per_row,
                   int index_bits, uint64_t* batch_size_out, char* err, size_t err_len);
/* Inverse of dbm_batch_size: a budget that yields `batch_size` rows. */
uint64_t dbm_max_bytes_for_batch_size(int64_t n, int k, int l, uint64_t batch_size, int backend,
                                      int64_t neigh_per_row, int index_bits);
/* The reference's per-batch route rule: 1 = annotate (sparse), 0 = dense. */
int dbm_annotate_pays(int64_t nnz, int64_t pairs, int k, int64_t d);
/* Index width the reference's --index auto would pick for n (32 or 64). */
int dbm_auto_index_bits(int64_t n);

/* ---- build identity ------------------------------------------------------------------ */
/* Static JSON object: git_sha, build_id, cuda_arch, configured_backend, compiled_backends. */
const char* dbm_build_info_json(void);

#ifdef __cplusplus
}
#endif

#endif /* DBM_H */
