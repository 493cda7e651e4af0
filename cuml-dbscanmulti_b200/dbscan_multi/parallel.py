"""Multi-GPU fit_multi: one process per GPU, torch.distributed for the exchanges.

The reference's fit_multi is single-GPU (runner_multi.cuh:15-16 removed cuML's multi-node
path).  Here the work shards without changing a single label:

1. every rank evaluates its share of the 128 x 128 tile pairs (i <= j; runs of 64 work items
   dealt round-robin, so the shares cost alike) of the distance pass (``dbm_distance_shard``):
   per-code histograms for all N rows and the neighbour pairs found in its share;
2. the histograms are summed across ranks (all-reduce) -- exact degrees everywhere -- and the
   neighbour pairs are all-gathered (variable counts, padded);
3. every rank labels a contiguous range of the k*l configurations from the complete graph
   (``dbm_fit_multi_from_graph``), with a batch plan that is identical on all ranks because the
   budget and the CSR memory cap are agreed first (minimum over ranks); the ranges balance the
   neighbour entries of the configs' eps rather than the config count;
4. the label rows are all-gathered (in place when the configs split evenly), so every rank ends
   with the full (k*l, N) result.

The collectives run on whatever backend the process group has (NCCL over NVLink on B200s,
gloo for the CPU tests).  The kernel work sits behind a ``stages`` object so the tests can
drive this exact orchestration with an oracle-backed fake on CPU ranks.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from . import (DBM_OK, DbmError, DbscanMulti, FitResult, Options, Stats, ROUTE_NAMES, BACKENDS,
               INDEX, ROUTES, normalize_eps, normalize_min_samples, stream_arg)

TILE = 128


SHARD_RUN = 64  # kShardRun of dbm_internal.cuh


def shard_items(total: int, shard: int, nshards: int) -> np.ndarray:
    """The global indices of the work items a shard evaluates, in its local order (the rule of
    dbm_internal.cuh shard_item / shard_items): runs of SHARD_RUN consecutive items dealt
    round-robin over the shards."""
    i = np.arange(total, dtype=np.int64)
    g = ((i // SHARD_RUN) * nshards + shard) * SHARD_RUN + i % SHARD_RUN
    return g[g < total]


def tile_pair_indices(n: int, shard: int, nshards: int) -> np.ndarray:
    """The tile-pair indices (i <= j, triangle order) a shard evaluates when no worklist is
    built (n < 4096: no pruning)."""
    t = (n + TILE - 1) // TILE
    return shard_items(t * (t + 1) // 2, shard, nshards)


def config_range(c: int, rank: int, world: int) -> tuple[int, int]:
    return c * rank // world, c * (rank + 1) // world


# Per-element costs of the labelling kernels in ns, fitted to C4 config-range timings on one
# GPU (dbm_fit_multi_from_graph; 8 batches, 3.84e6 max-eps entries): sparse batches walk the
# max-eps entries with their codes, so every rank that owns a config pays one walk of them
# (~0.13 ms) whatever its eps; the union per (entry of the config's eps, owned config), ~0.045 ms
# per 1e6; the relabel per (point, owned config), ~0.013 ms per 1e6.  The per-rank fixed part
# (~0.45 ms of launches and initialisation) is the same on every rank and does not move the split.
LABEL_COST_WALK = 0.034
LABEL_COST_UNION = 0.045
LABEL_COST_RELABEL = 0.0134


class _LabelCost:
    """The labelling cost model with prefix sums, so the cost of any config range is O(1)."""

    def __init__(self, per_eps: list[float], l: int, n: int):
        self.l, self.n, self.k = int(l), int(n), len(per_eps)
        self.last = float(per_eps[-1]) if per_eps else 0.0
        per_cfg = np.repeat(np.asarray(per_eps, dtype=np.float64), self.l)
        self.cfg_pre = np.concatenate([[0.0], np.cumsum(per_cfg)])

    def __call__(self, a: int, b: int) -> float:
        if b <= a:
            return 0.0
        union = self.cfg_pre[b] - self.cfg_pre[a]
        return float(LABEL_COST_WALK * self.last + LABEL_COST_UNION * union
                     + LABEL_COST_RELABEL * self.n * (b - a))


def labelling_cost(per_eps: list[float], l: int, n: int, a: int, b: int) -> float:
    """Model cost of labelling the configs [a, b) (eps-major, l per eps)."""
    return _LabelCost(per_eps, l, n)(a, b)


def labelling_ranges(per_eps: list[float], l: int, n: int, world: int) -> list[tuple[int, int]]:
    """Contiguous config ranges, one per rank, minimising the largest modelled labelling cost
    (bisection on the bound with a greedy feasibility sweep; the cost of a range only grows as
    it widens).  Every rank that owns a config walks the max-eps entries once; the unions scale
    with the entries of each owned config's eps, so the largest eps's configs are spread over
    ranks.  Deterministic: every rank computes the same split from the same (all-reduced) entry
    counts."""
    c = len(per_eps) * l
    if world <= 1 or c == 0:
        return [(0, c)] + [(c, c)] * max(0, world - 1)
    cost = _LabelCost(per_eps, l, n)

    def sweep(bound):
        out, a = [], 0
        while a < c:
            b = a + 1
            while b < c and cost(a, b + 1) <= bound:
                b += 1
            out.append((a, b))
            a = b
            if len(out) > world:  # infeasible already
                break
        return out

    lo = max(cost(i, i + 1) for i in range(c))
    hi = cost(0, c)
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        r = sweep(mid)
        if len(r) <= world and r[-1][1] == c:
            hi = mid
        else:
            lo = mid
    ranges = sweep(hi)
    # every rank gets work while configs remain: split the costliest multi-config range in two
    while len(ranges) < min(world, c):
        i = max((j for j in range(len(ranges)) if ranges[j][1] - ranges[j][0] > 1),
                key=lambda j: (cost(*ranges[j]), -j))
        a, b = ranges[i]
        best = min(range(a + 1, b), key=lambda s: (max(cost(a, s), cost(s, b)), s))
        ranges[i:i + 1] = [(a, best), (best, b)]
    return ranges + [(c, c)] * (world - len(ranges))


class DeviceStages:
    """The C-ABI stages on this rank's GPU.  With a process group of several ranks, the distance
    stage shards the prune's bound pass by work units and all-gathers the per-unit counts and keep
    masks over the group (``group=None``: the default group)."""

    def __init__(self, handle: DbscanMulti, group=None):
        self.h = handle
        self.lib = handle._lib
        self.group = group
        self.last_shard_stats: dict[str, Any] = {}
        self._prune_bufs = None

    def _mem_info(self) -> tuple[int, int]:
        """(free, total) device memory, queried at most once a second (the query costs
        milliseconds of host time)."""
        import time

        import torch

        now = time.monotonic()
        if getattr(self, "_mem_at", None) is None or now - self._mem_at > 1.0:
            self._mem = tuple(int(v) for v in torch.cuda.mem_get_info(self.h.device))
            self._mem_at = now
        return self._mem

    def default_budget(self) -> int:
        """80% of (free + this handle's reusable workspace), as the reference's fit_multi."""
        free, total = self._mem_info()
        reusable = self.h.workspace_bytes
        used = total - min(total, free)
        available = total if reusable > used else min(total, free + reusable)
        return 80 * available // 100

    def free_bytes(self) -> int:
        """Free device memory for the CSR-fits check (the workspace is reused across calls)."""
        return self._mem_info()[0]

    def _gathered_prune(self, x, eps: np.ndarray, shard: int, nshards: int, s: int):
        """This rank bounds its equal share of the prune units; one all-gather of the counts and
        one of the keep masks give every rank all of them.  None when there is no prune (N < 4096),
        a single shard, or no process group of nshards ranks (shards driven from one process)."""
        import torch
        import torch.distributed as dist

        n, d = int(x.shape[0]), int(x.shape[1])
        units = int(self.lib.dbm_prune_units(n))
        if (nshards <= 1 or units == 0 or not dist.is_available() or not dist.is_initialized()
                or dist.get_world_size(self.group) != nshards):
            return None
        words = int(self.lib.dbm_prune_mask_words())
        chunk = -(-units // nshards)
        # one int32 buffer per rank slot: [chunk counts | chunk * words mask words], so a single
        # all-gather exchanges both; the counts and masks of all units are then strided views
        per = chunk * (1 + words)
        if self._prune_bufs is None or self._prune_bufs[0].numel() != nshards * per or \
                self._prune_bufs[0].device != x.device:
            gathered = torch.zeros(nshards * per, dtype=torch.int32, device=x.device)
            counts = torch.zeros(nshards * chunk, dtype=torch.int32, device=x.device)
            masks = torch.zeros(nshards * chunk * words, dtype=torch.int32, device=x.device)
            self._prune_bufs = (gathered, counts, masks)
        gathered, counts, masks = self._prune_bufs
        u0, u1 = min(units, shard * chunk), min(units, (shard + 1) * chunk)
        err = ctypes.create_string_buffer(1024)
        rc = self.lib.dbm_distance_prune_units(self.h._h, ctypes.c_void_p(x.data_ptr()), n, d,
                                               eps.ctypes.data_as(ctypes.c_void_p), len(eps), u0, u1,
                                               ctypes.c_void_p(counts.data_ptr()), ctypes.c_void_p(masks.data_ptr()),
                                               stream_arg(s), err, len(err))
        if rc != DBM_OK:
            raise DbmError(rc, err.value.decode())
        mine = torch.cat([counts[shard * chunk:(shard + 1) * chunk],
                          masks[shard * chunk * words:(shard + 1) * chunk * words]])
        dist.all_gather_into_tensor(gathered, mine, group=self.group)
        g = gathered.view(nshards, per)
        counts.view(nshards, chunk).copy_(g[:, :chunk])
        masks.view(nshards, chunk * words).copy_(g[:, chunk:])
        return counts, masks

    def distance_shard(self, x, eps: np.ndarray, shard: int, nshards: int, cap_hint: int):
        import torch

        n, d = int(x.shape[0]), int(x.shape[1])
        k = len(eps)
        hist = torch.empty((k, n), dtype=torch.int32, device=x.device)
        cap = max(int(cap_hint), 1024)
        s = torch.cuda.current_stream(x.device).cuda_stream
        err = ctypes.create_string_buffer(1024)
        pruned = self._gathered_prune(x, eps, shard, nshards, s)
        for _ in range(2):
            edges = torch.empty(cap, dtype=torch.int64, device=x.device)
            found = ctypes.c_uint64(0)
            st = Stats()
            if pruned is not None:
                rc = self.lib.dbm_distance_shard_pruned(
                    self.h._h, ctypes.c_void_p(x.data_ptr()), n, d, eps.ctypes.data_as(ctypes.c_void_p), k, shard,
                    nshards, ctypes.c_void_p(pruned[0].data_ptr()), ctypes.c_void_p(pruned[1].data_ptr()),
                    ctypes.c_void_p(hist.data_ptr()), ctypes.c_void_p(edges.data_ptr()), cap, ctypes.byref(found),
                    ctypes.byref(st), stream_arg(s), err, len(err))
            else:
                rc = self.lib.dbm_distance_shard(self.h._h, ctypes.c_void_p(x.data_ptr()), n, d,
                                                 eps.ctypes.data_as(ctypes.c_void_p), k, shard, nshards,
                                                 ctypes.c_void_p(hist.data_ptr()), ctypes.c_void_p(edges.data_ptr()),
                                                 cap, ctypes.byref(found), ctypes.byref(st), stream_arg(s), err,
                                                 len(err))
            if rc != DBM_OK:
                raise DbmError(rc, err.value.decode())
            self.last_shard_stats = st.as_dict()
            if found.value <= cap:
                return hist, edges[: found.value]
            cap = int(found.value)
        raise DbmError(-5, "neighbour-pair buffer overflowed twice")

    def fit_from_graph(self, n, d, eps, ms, hist, edges, cfg_begin, cfg_end, opt: Options):
        import torch

        k, l = len(eps), len(ms)
        labels = torch.empty((k * l, n), dtype=torch.int32, device=hist.device)
        st = Stats()
        routes = self.h._routes_buffer(n + 1)
        s = torch.cuda.current_stream(hist.device).cuda_stream
        err = ctypes.create_string_buffer(1024)
        edges = edges.contiguous()
        rc = self.lib.dbm_fit_multi_from_graph(
            self.h._h, n, d, eps.ctypes.data_as(ctypes.c_void_p), k, ms.ctypes.data_as(ctypes.c_void_p), l,
            ctypes.c_void_p(hist.data_ptr()), ctypes.c_void_p(edges.data_ptr()) if edges.numel() else None,
            int(edges.numel()), cfg_begin, cfg_end, ctypes.c_void_p(labels.data_ptr()), None,
            ctypes.byref(opt), ctypes.byref(st), routes, n + 1, stream_arg(s), err, len(err))
        if rc != DBM_OK:
            raise DbmError(rc, err.value.decode())
        return labels, st.as_dict(), [ROUTE_NAMES[int(routes[i])] for i in range(int(st.batches))]


def _all_gather_varlen(dist, t, group, extra=None):
    """All-gather 1-D tensors of different lengths: one exchange of the counts, then one flat
    all_gather of buffers padded to the longest; returns the parts.  `extra`, a tensor already
    queued on the stream, is copied to the host in the same synchronisation as the counts and
    returned with the parts (or None)."""
    import torch

    world = dist.get_world_size(group)
    cnt = torch.tensor([t.numel()], dtype=torch.int64, device=t.device)
    counts_t = torch.zeros(world, dtype=torch.int64, device=t.device)
    dist.all_gather_into_tensor(counts_t, cnt, group=group)
    host = counts_t.cpu()
    extra_host = extra.cpu() if extra is not None else None
    counts = [int(c) for c in host.tolist()]
    mx = max(max(counts), 1)
    buf = torch.empty(mx, dtype=t.dtype, device=t.device)
    buf[: t.numel()] = t
    out = torch.empty(world * mx, dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    parts = [out[r * mx: r * mx + c] for r, c in enumerate(counts)]
    return (parts, extra_host) if extra is not None else parts


def _gather_config_rows(dist, labels, C: int, n: int, group, ranges=None):
    """Every rank holds the rows ranges[r] (default config_range(C, r, world)) of a (C, n) label
    matrix; returns the full matrix on every rank.  The row counts are known on every rank (no
    count exchange); with equal shares the gather is in place into `labels` itself, else through
    a padded buffer."""
    import torch

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if ranges is None:
        ranges = [config_range(C, r, world) for r in range(world)]
    sizes = [b - a for a, b in ranges]
    if min(sizes) == max(sizes):
        flat = labels.reshape(-1)
        per = sizes[0] * n
        dist.all_gather_into_tensor(flat, flat[rank * per:(rank + 1) * per], group=group)
        return labels
    mx = max(sizes)
    a, b = ranges[rank]
    send = torch.empty((mx, n), dtype=labels.dtype, device=labels.device)  # rows past b - a are never read
    send[: b - a] = labels[a:b]
    out = torch.empty((world * mx, n), dtype=labels.dtype, device=labels.device)
    dist.all_gather_into_tensor(out, send, group=group)
    return torch.cat([out[r * mx: r * mx + sizes[r]] for r in range(world)])


def agree_limits(stages, max_bytes_per_batch: int = 0, csr_cap_bytes: int = 0, group=None, device=None):
    """The budget and the CSR memory cap every rank will use (minimum over ranks), so that all
    ranks compute the same batch plan.  One collective and one host synchronisation: callers that
    fit repeatedly compute it once and pass it to sharded_fit_multi(limits=...)."""
    import torch
    import torch.distributed as dist

    agree = torch.tensor([max_bytes_per_batch or stages.default_budget(), csr_cap_bytes or stages.free_bytes()],
                         dtype=torch.int64, device=device)
    dist.all_reduce(agree, op=dist.ReduceOp.MIN, group=group)
    return int(agree[0].item()), int(agree[1].item())


def gather_points(x_host, device, group=None, out=None):
    """Host points -> the full (N, D) float32 tensor on every rank's device: rank r copies only its
    row slice [N r / G, N (r + 1) / G) from (pinned) host memory, then one all-gather over the
    process group (NVLink on B200s) assembles the rest, instead of every rank copying all N rows
    across PCIe.  `out` (>= G * ceil(N / G) rows) is reused when given."""
    import torch
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    xh = x_host if type(x_host).__module__.startswith("torch") else torch.from_numpy(np.ascontiguousarray(x_host, np.float32))
    n, d = int(xh.shape[0]), int(xh.shape[1])
    chunk = -(-n // world)
    if out is None or out.shape[0] < world * chunk or out.shape[1] != d:
        out = torch.empty((world * chunk, d), dtype=torch.float32, device=device)
    buf = out[: world * chunk]
    a, b = min(n, rank * chunk), min(n, (rank + 1) * chunk)
    mine = buf[rank * chunk:(rank + 1) * chunk]
    if b > a:
        mine[: b - a].copy_(xh[a:b], non_blocking=True)
    dist.all_gather_into_tensor(buf, mine, group=group)
    return buf[:n], out


def sharded_fit_multi(stages, x, eps, min_samples, *, group=None, max_bytes_per_batch: int = 0,
                      backend: str = "cuvs", index: str = "auto", route: str = "auto",
                      neigh_per_row: int = 0, csr_cap_bytes: int = 0, limits=None,
                      device=None) -> FitResult:
    """fit_multi over all ranks of ``group``; every rank returns the full (k*l, N) labels.

    ``x`` is the (N, D) float32 tensor present on every rank; with ``device`` set, ``x`` is the
    host copy (NumPy array or CPU tensor, pinned for asynchronous copies) and gather_points puts
    it on ``device`` (each rank copies 1/G of the rows, one all-gather assembles the rest).
    ``limits`` = agree_limits(...) skips the per-call agreement of the budget and CSR cap."""
    import torch
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    e = normalize_eps(eps)
    m = normalize_min_samples(min_samples)
    k, l = len(e), len(m)
    if backend not in BACKENDS or index not in INDEX or route not in ROUTES:
        raise DbmError(-1, "unknown backend, index or route")
    if route != "auto" and backend != "cuvs":
        raise DbmError(-1, "--route only applies to the cuvs backend")
    if device is not None:
        x, stages._points_buf = gather_points(x, device, group, getattr(stages, "_points_buf", None))
    n, d = int(x.shape[0]), int(x.shape[1])
    dev = x.device

    # identical batch plans on every rank: agree on the budget and the CSR memory cap
    budget, cap = limits if limits is not None else agree_limits(stages, max_bytes_per_batch, csr_cap_bytes,
                                                                 group, dev)
    opt = Options(BACKENDS[backend], INDEX[index], ROUTES[route], int(neigh_per_row), budget, cap)

    hint = n * (neigh_per_row if neigh_per_row > 0 else 16) // (2 * world) + 1024
    hist, edges = stages.distance_shard(x, e, rank, world, hint)
    dist.all_reduce(hist, op=dist.ReduceOp.SUM, group=group)
    # per-eps entry counts ride along with the pair counts' host synchronisation
    per_eps_dev = hist.to(torch.int64).cumsum(0).sum(1)
    parts, per_eps_host = _all_gather_varlen(dist, edges, group, extra=per_eps_dev)
    all_edges = torch.cat(parts) if parts else edges

    # configs split by modelled labelling cost: the slab walks of each eps a rank touches, the
    # union per owned config and the relabel, from the per-eps entry counts (known identically
    # on every rank from the summed histograms)
    per_eps = [float(v) for v in per_eps_host.tolist()]
    ranges = labelling_ranges(per_eps, l, n, world)
    c0, c1 = ranges[rank]
    if c1 > c0:
        labels, stats, routes = stages.fit_from_graph(n, d, e, m, hist, all_edges, c0, c1, opt)
    else:  # more ranks than configs: nothing to label here
        labels, stats, routes = torch.empty((k * l, n), dtype=torch.int32, device=hist.device), {}, []
    full = _gather_config_rows(dist, labels, k * l, n, group, ranges)
    stats = dict(stats)
    stats["world_size"] = world
    stats["edges"] = int(all_edges.numel())
    return FitResult(labels=full, core=None, eps=e, min_samples=m, stats=stats, batch_routes=routes,
                     index="int64" if stats.get("index_bits") == 64 else "int32", backend=backend)
