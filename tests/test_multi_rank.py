"""Multi-rank orchestration on CPU: gloo process groups (world size 2 and 3) run the real
``dbscan_multi.parallel.sharded_fit_multi`` with an oracle-backed stand-in for the two
device stages.  Checked: the tile-pair shards partition the triangle exactly, the summed
histograms and gathered neighbour pairs equal the single-process graph, budget and CSR cap
are agreed (minimum over ranks), every rank ends with the full, oracle-identical labels."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import batching
import oracle
from dbscan_multi import parallel

TILE = parallel.TILE


def tri_coords(c):
    j = int((np.sqrt(8.0 * c + 1.0) - 1.0) * 0.5)
    while j * (j + 1) // 2 > c:
        j -= 1
    while (j + 1) * (j + 2) // 2 <= c:
        j += 1
    return c - j * (j + 1) // 2, j


def make_points(seed=4, n=700):
    rng = np.random.default_rng(seed)
    c = rng.uniform(-3, 3, size=(5, 2))
    pts = c[rng.integers(0, 5, n - 60)] + rng.normal(0, 0.35, (n - 60, 2))
    return np.vstack([pts, rng.uniform(-3, 3, (60, 2))]).astype(np.float32)


EPS = [0.15, 0.25, 0.35]
MS = [3, 6]


class OracleStages:
    """CPU stand-in for the C-ABI stages, computed from the oracle's per-pair codes."""

    def __init__(self, pts, rank):
        self.pts = pts
        self.rank = rank
        self.codes, self.deg = oracle.codes_degrees(pts, EPS)
        self.seen_opt = None

    def default_budget(self):
        # ~150-row batches; ranks disagree and the minimum must win
        return batching.max_bytes_for_batch_size(700, 3, 2, 150, True, 0, 32) + 1000 * self.rank

    def free_bytes(self):
        return 10**9 - self.rank

    def distance_shard(self, x, eps, shard, nshards, cap_hint):
        n = len(self.pts)
        k = len(eps)
        mine = parallel.tile_pair_indices(n, shard, nshards)
        hist = np.zeros((k, n), np.int32)
        words = []
        for c in mine.tolist():
            ti, tj = tri_coords(c)
            for i in range(ti * TILE, min(n, ti * TILE + TILE)):
                for j in range(tj * TILE, min(n, tj * TILE + TILE)):
                    if ti == tj and j <= i:
                        continue
                    code = int(self.codes[i, j])
                    if code == 255:
                        continue
                    hist[code, i] += 1
                    hist[code, j] += 1
                    words.append((i << 32) | (code << 28) | j)
        return torch.from_numpy(hist), torch.tensor(words, dtype=torch.int64)

    def fit_from_graph(self, n, d, eps, ms, hist, edges, c0, c1, opt):
        k, l = len(eps), len(ms)
        # complete graph check: cumulative histograms are the oracle's degrees
        deg = 1 + np.cumsum(hist.numpy(), axis=0)
        assert np.array_equal(deg, self.deg)
        iu, ju = np.nonzero(np.triu(self.codes != 255, 1))
        want = set(((iu.astype(np.int64) << 32) | (self.codes[iu, ju].astype(np.int64) << 28) | ju).tolist())
        got = edges.numpy().tolist()
        assert len(got) == len(want) and set(got) == want
        self.seen_opt = (opt.max_bytes_per_batch, opt.csr_cap_bytes)
        bs = batching.compute_batch_size(n, k, l, opt.max_bytes_per_batch, True, 0, 32)
        lab, _, _ = oracle.fit_multi(self.pts, eps, ms, bs)
        out = np.full((k * l, n), -7, np.int32)
        out[c0:c1] = lab[c0:c1]
        return torch.from_numpy(out), {"batches": (n + bs - 1) // bs, "index_bits": 32}, []


def _worker(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pts = make_points()
        st = OracleStages(pts, rank)
        res = parallel.sharded_fit_multi(st, torch.from_numpy(pts), EPS, MS, index="int32")
        np.save(os.path.join(result_dir, f"labels_{rank}.npy"), res.labels.numpy())
        np.save(os.path.join(result_dir, f"opt_{rank}.npy"), np.asarray(st.seen_opt, dtype=np.int64))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tile_pair_shards_partition_the_triangle():
    for n in (1, 127, 128, 129, 1000, 4097, 40000):
        t = (n + TILE - 1) // TILE
        for world in (1, 2, 3, 8):
            parts = [parallel.tile_pair_indices(n, r, world) for r in range(world)]
            allp = np.sort(np.concatenate(parts))
            assert np.array_equal(allp, np.arange(t * (t + 1) // 2))  # every tile pair exactly once
            # runs of consecutive items stay together, and the shares differ by at most one run
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= parallel.SHARD_RUN
            for p in parts:
                assert np.all(np.diff(p)[np.arange(len(p) - 1) % parallel.SHARD_RUN != parallel.SHARD_RUN - 1] == 1)
    assert [parallel.config_range(16, r, 8) for r in range(8)] == [(2 * r, 2 * r + 2) for r in range(8)]
    for c in (1, 5, 9, 16, 100):
        for world in (1, 2, 3, 8):
            rs = [parallel.config_range(c, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == c and all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_fit_on_gloo_ranks_equals_single_process(tmp_path, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    pts = make_points()
    opt0 = np.load(tmp_path / "opt_0.npy")
    assert opt0[0] == batching.max_bytes_for_batch_size(700, 3, 2, 150, True, 0, 32)  # minimum over ranks
    assert opt0[1] == 10**9 - (world - 1)
    bs = batching.compute_batch_size(len(pts), len(EPS), len(MS), int(opt0[0]), True, 0, 32)
    assert bs == 150  # the agreed budget really batches
    want, _, _ = oracle.fit_multi(pts, EPS, MS, bs)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"labels_{r}.npy"), want)
        assert np.array_equal(np.load(tmp_path / f"opt_{r}.npy"), opt0)


class FailingStages(OracleStages):
    """Rank 1 fails inside its distance stage (an injected host-side fault)."""

    def distance_shard(self, x, eps, shard, nshards, cap_hint):
        if self.rank == 1:
            raise RuntimeError("injected failure on rank 1")
        return super().distance_shard(x, eps, shard, nshards, cap_hint)


def _failing_worker(rank, world, port, result_dir):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    outcome = "ok"
    try:
        parallel.sharded_fit_multi(FailingStages(make_points(), rank), torch.from_numpy(make_points()), EPS, MS)
    except Exception as exc:  # the failing rank raises; the survivor's collective times out
        outcome = type(exc).__name__ + ": " + str(exc)[:200]
    with open(os.path.join(result_dir, f"outcome_{rank}.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)  # leave without a final barrier on the broken group


def test_a_failing_rank_is_detected_by_the_others(tmp_path):
    """Failure detection across ranks on the host: rank 1 raises before its collectives; rank 0
    must come back with an error from its next collective (process-group timeout) instead of
    hanging, and both processes exit."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    o0 = (tmp_path / "outcome_0.txt").read_text()
    o1 = (tmp_path / "outcome_1.txt").read_text()
    assert "injected failure" in o1
    assert o0 != "ok"


def _gather_worker(rank, world, port, C, n, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b = parallel.config_range(C, rank, world)
        labels = torch.full((C, n), -9, dtype=torch.int32)
        labels[a:b] = torch.arange(a * n, b * n, dtype=torch.int32).reshape(b - a, n)
        full = parallel._gather_config_rows(dist, labels, C, n, None)
        np.save(os.path.join(result_dir, f"rows_{rank}.npy"), full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("C,world", [(5, 2), (7, 3), (6, 3), (1, 2)])
def test_label_rows_gather_even_and_uneven_splits(tmp_path, C, world):
    n = 11
    mp.spawn(_gather_worker, args=(world, _free_port(), C, n, str(tmp_path)), nprocs=world, join=True)
    want = np.arange(C * n, dtype=np.int32).reshape(C, n)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"rows_{r}.npy"), want)


def _brute_force_best(per_eps, l, n, world):
    import itertools

    c = len(per_eps) * l
    best = None
    for cuts in itertools.combinations(range(1, c), min(world, c) - 1):
        bounds = (0,) + cuts + (c,)
        worst = max(parallel.labelling_cost(per_eps, l, n, a, b) for a, b in zip(bounds, bounds[1:]))
        best = worst if best is None else min(best, worst)
    return best


def test_labelling_ranges_partition_and_match_the_brute_force_optimum():
    rng = np.random.default_rng(8)
    for k, l in ((1, 5), (3, 2), (4, 4), (5, 1)):
        for world in (1, 2, 3, 4, 8):
            per_eps = sorted(float(v) for v in rng.uniform(0, 1e6, k))  # nested eps: counts grow
            n = 100_000
            rs = parallel.labelling_ranges(per_eps, l, n, world)
            c = k * l
            assert len(rs) == world and rs[0][0] == 0 and rs[-1][1] == c
            assert all(a[1] == b[0] and a[0] <= a[1] for a, b in zip(rs, rs[1:]))
            if c >= world:
                assert all(b > a for a, b in rs)
            got = max(parallel.labelling_cost(per_eps, l, n, a, b) for a, b in rs)
            assert got <= _brute_force_best(per_eps, l, n, world) * (1 + 1e-9)
    # identical on every rank: a pure function of its inputs
    pe = [250.0, 19000.0, 371500.0, 3862750.0]
    assert parallel.labelling_ranges(pe, 4, 10**6, 8) == parallel.labelling_ranges(list(pe), 4, 10**6, 8)


def test_labelling_ranges_scale_to_large_grids():
    """16 eps x 100 minPts = 1600 configs over 8 ranks: the split is computed in well under a
    second (every rank computes it inside each sharded fit)."""
    import time

    per_eps = [float(1e4 * (1.7 ** e)) for e in range(16)]
    t0 = time.perf_counter()
    rs = parallel.labelling_ranges(per_eps, 100, 1_000_000, 8)
    assert time.perf_counter() - t0 < 1.0
    assert len(rs) == 8 and rs[0][0] == 0 and rs[-1][1] == 1600 and all(b > a for a, b in rs)


def _points_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        from dbscan_multi import parallel

        pts = make_points()
        out = None
        for _ in range(2):  # the second call reuses the buffer
            full, out = parallel.gather_points(torch.from_numpy(pts), torch.device("cpu"), out=out)
        budget, cap = parallel.agree_limits(_LimitStages(rank), 0, 0, device=torch.device("cpu"))
        np.save(os.path.join(result_dir, f"g{rank}.npy"), full.numpy())
        np.save(os.path.join(result_dir, f"l{rank}.npy"), np.array([budget, cap]))
    finally:
        dist.destroy_process_group()


class _LimitStages:
    """Per-rank free-memory figures differ; the agreed limits must be the minimum over ranks."""

    def __init__(self, rank):
        self.rank = rank

    def default_budget(self):
        return 1000 + 10 * self.rank

    def free_bytes(self):
        return 500 - self.rank


@pytest.mark.parametrize("world", [2, 3])
def test_points_gathered_from_host_slices_and_limits_agreed(tmp_path, world):
    """gather_points: each rank copies only its row slice, one all-gather assembles the rest,
    identical to the host array on every rank (N not a multiple of the world size); agree_limits:
    the minimum budget and cap over ranks, identical everywhere."""
    import torch.multiprocessing as mp

    port = _free_port()
    mp.spawn(_points_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    pts = make_points()
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"g{r}.npy"), pts)
        assert list(np.load(tmp_path / f"l{r}.npy")) == [1000, 500 - (world - 1)]


def test_labelling_split_spreads_the_largest_eps_configs():
    """C4's per-eps entry counts (almost every entry belongs to the largest eps): every rank walks
    the max-eps entries once whatever it owns, so the split spreads the largest eps's configs,
    whose unions dominate, over the ranks instead of giving them all to one."""
    pe = [394.0, 17668.0, 357400.0, 3840788.0]
    for world in (2, 4, 8):
        rs = parallel.labelling_ranges(pe, 4, 10**6, world)
        owners = [r for r, (a, b) in enumerate(rs) if any(12 <= c < 16 for c in range(a, b))]
        assert len(owners) >= min(world, 4) // 2 + 1, (world, rs)
