"""GPU parity: the CUDA path (through the C ABI) against the reference's goldens and the oracle.

Bar: raw equality of every label (int32) and core mask, and of the per-eps degrees, for the
same float32 input and the same batch partition.  Cases follow the reference's own tests:
the 13 adversarial golden bundles in every mode of the reference binary
(tools/run_validation_matrix.py:309-320), the selftest's recorded answers and checks
(src/main.cu:958-1357), plus seeded random grids against the oracle, batch-partition
adversarial cases, and full-size properties on row samples.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import batching
import dbscan_multi as dm
import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("0*.npz"))


@pytest.fixture(scope="module")
def torch_mod():
    import torch

    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def h(torch_mod):
    handle = dm.DbscanMulti(0)
    yield handle
    handle.close()


def gpu_fit(h, torch, pts, eps, ms, **kw):
    x = torch.from_numpy(np.ascontiguousarray(pts, dtype=np.float32)).to("cuda:0")
    r = h.fit_multi(x, eps, ms, return_core=True, **kw)
    return r.labels.cpu().numpy(), r.core.cpu().numpy().astype(bool), r


def load_case(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return z["points"], z["eps"].astype(np.float32), z["min_samples"].astype(np.int32), z["labels"]


MODES = {
    "cuvs_auto_i32": dict(backend="cuvs", index="int32"),
    "cuvs_annotated_i32": dict(backend="cuvs", index="int32", route="annotated"),
    "cuvs_dense_i32": dict(backend="cuvs", index="int32", route="dense"),
    "cuvs_auto_i64": dict(backend="cuvs", index="int64"),
    "codes_i32": dict(backend="codes", index="int32"),
    "codes_i64": dict(backend="codes", index="int64"),
    "cuvs_batched": dict(backend="cuvs", index="int32", max_bytes_per_batch=1_000_000),
    "codes_batched": dict(backend="codes", index="int32", max_bytes_per_batch=1_000_000),
}


@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("name", CASES)
def test_golden_bundle_every_mode(h, torch_mod, name, mode):
    pts, eps, ms, expected = load_case(name)
    labels, core, r = gpu_fit(h, torch_mod, pts, eps, ms, **MODES[mode])
    assert np.array_equal(labels, expected), f"{name}/{mode}"
    _, ocore, _ = oracle.fit_multi(pts, eps, ms)
    assert np.array_equal(core, ocore)
    if name == "009_forced_batches_2d" and mode == "cuvs_batched":
        assert r.stats["batches"] == 11 and r.stats["batch_size"] == 98
    if name == "009_forced_batches_2d" and mode == "codes_batched":
        assert r.stats["batches"] == 7 and r.stats["batch_size"] == 164
    if MODES[mode].get("route") in ("annotated", "dense") and len(eps) > 1:
        assert set(r.batch_routes) == {MODES[mode]["route"]}


def test_golden_bundles_host_path(h):
    for name in CASES:
        pts, eps, ms, expected = load_case(name)
        r = h.fit_multi(pts, eps, ms)
        assert isinstance(r.labels, np.ndarray)
        assert np.array_equal(r.labels, expected), name


def test_selftest_known_answers(h, torch_mod):
    spec = json.loads((GOLDEN / "selftest_answers.json").read_text())
    pts = oracle.selftest_points(1000, 2, 42)
    labels, _, r = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], index="int32")
    for cfg, ans in enumerate(spec["configurations"]):
        assert int(labels[cfg].max()) + 1 == ans["clusters"]
        assert int((labels[cfg] < 0).sum()) == ans["noise"]
    # forced 4 x 750 batches (selftest part 2)
    budget = dm.max_bytes_for_batch_size(3000, 3, 3, 750, "cuvs", 0, "int32")
    lb, _, rb = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], index="int32",
                        max_bytes_per_batch=budget)
    assert rb.stats["batches"] == spec["forced_batches"] == 4
    assert np.array_equal(lb, labels)
    # codes backend, three repetitions, deterministic (part 1)
    for _ in range(3):
        lc, _, _ = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], backend="codes")
        assert np.array_equal(lc, labels)
    # int32 == int64 (part 4)
    li, _, _ = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], index="int64")
    assert np.array_equal(li, labels)
    # routes forced both ways (part 6)
    for route in ("annotated", "dense"):
        lr, _, rr = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], route=route)
        assert np.array_equal(lr, labels) and set(rr.batch_routes) == {route}


def test_selftest_batch_correction(h, torch_mod):
    """neigh_per_row lies (1) under a 1 MB CSR cap: the batch must be corrected, labels equal
    (selftest part 5, src/main.cu:1238-1281)."""
    spec = json.loads((GOLDEN / "selftest_answers.json").read_text())
    pts = oracle.selftest_points(1000, 2, 42)
    ref, _, _ = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], index="int32")
    lab, _, r = gpu_fit(h, torch_mod, pts, spec["eps"], spec["min_samples"], index="int32",
                        neigh_per_row=1, csr_cap_bytes=1024 * 1024)
    assert r.stats["batch_corrections"] > 0
    assert np.array_equal(lab, ref)
    # the batch size after correction follows the reference's rule, replayed on the oracle
    _, _, deg = oracle.fit_multi(pts, spec["eps"], spec["min_samples"])
    bs, attempts, corrections = batching.plan(3000, 3, 3, r.stats["max_bytes_per_batch"], deg[-1], deg,
                                              True, 1, 32, 1024 * 1024)
    assert (bs, attempts, corrections) == (r.stats["batch_size"], r.stats["attempts"], r.stats["batch_corrections"])
    ob, _, _ = oracle.fit_multi(pts, spec["eps"], spec["min_samples"], bs)
    assert np.array_equal(lab, ob)


@pytest.mark.parametrize("d", [2, 8, 16, 32, 33])
def test_selftest_dimension_sweep(h, torch_mod, d):
    pts = oracle.selftest_points(500, d, 42)
    for eps in ([0.8], [0.3, 0.5, 0.8], [0.2, 0.3, 0.5, 0.65, 0.8]):
        labels, _, _ = gpu_fit(h, torch_mod, pts, eps, [4])
        assert int(labels[-1].max()) + 1 == 3
        noise = [(labels[e] < 0).sum() for e in range(len(eps))]
        assert all(b <= a for a, b in zip(noise, noise[1:]))
        ol, _, _ = oracle.fit_multi(pts, eps, [4])
        assert np.array_equal(labels, ol)


def test_selftest_high_dimension_equivalence(h, torch_mod):
    """D=33 and D=8193 (two informative coordinates) give the same partition (part 3b)."""
    eps = [0.5, 1.0, 2.0, 3.0, 4.0]
    a, _, _ = gpu_fit(h, torch_mod, oracle.selftest_points(16, 33, 42), eps, [2], backend="codes")
    b, _, _ = gpu_fit(h, torch_mod, oracle.selftest_points(16, 8193, 42), eps, [2], backend="codes")
    assert np.array_equal(a, b)


def blobs(rng, n, d, centers, spread, noise_frac, box):
    c = rng.uniform(-box, box, size=(centers, d))
    m = n - int(noise_frac * n)
    assign = rng.integers(0, centers, size=m)
    pts = c[assign] + rng.normal(0, spread, size=(m, d))
    noise = rng.uniform(-box, box, size=(n - m, d))
    return np.vstack([pts, noise]).astype(np.float32)


RANDOM_CASES = [
    # n, d, k, l, seed, rows_per_batch (None = one batch)
    (1, 3, 2, 2, 0, None),
    (2, 1, 1, 1, 1, None),
    (127, 2, 3, 2, 2, None),
    (128, 4, 2, 3, 3, None),
    (129, 5, 4, 2, 4, 40),
    (1000, 2, 5, 3, 5, None),
    (1000, 3, 16, 4, 6, 123),
    (2049, 7, 3, 5, 7, 500),
    (3000, 16, 4, 4, 8, None),
    (3000, 31, 2, 2, 9, 700),
    (4097, 32, 3, 3, 10, None),
    (4097, 33, 4, 4, 11, 1000),
    (2500, 63, 2, 3, 12, None),
    (2500, 64, 3, 2, 13, 333),
    (2500, 65, 2, 2, 14, None),
    (1500, 129, 3, 2, 15, 256),
    (4500, 136, 2, 2, 19, 1500),  # ordered path with points wider than the shared-memory transpose
    (700, 300, 2, 2, 16, None),
    (9000, 8, 5, 1, 17, None),
    (9000, 2, 1, 5, 18, 2000),
]


@pytest.mark.parametrize("n,d,k,l,seed,rows", RANDOM_CASES)
def test_random_grid_matches_oracle(h, torch_mod, n, d, k, l, seed, rows):
    rng = np.random.default_rng(1000 + seed)
    pts = blobs(rng, n, d, centers=max(1, n // 300), spread=1.0, noise_frac=0.1, box=6.0)
    # eps spread around the typical intra-blob pair distance so every code is used
    base = float(np.sqrt(2.0 * d))
    eps = sorted({float(np.float32(base * f)) for f in np.linspace(0.35, 1.0, k)})
    ms = sorted({int(v) for v in np.unique(np.linspace(2, 30, l).astype(int))})
    kw = {}
    if rows is not None:
        kw["max_bytes_per_batch"] = dm.max_bytes_for_batch_size(n, len(eps), len(ms), rows, "cuvs")
    labels, core, r = gpu_fit(h, torch_mod, pts, eps, ms, **kw)
    bs = r.stats["batch_size"]
    if rows is not None:
        assert bs == min(rows, n)
    ol, ocore, odeg = oracle.fit_multi(pts, eps, ms, bs)
    assert np.array_equal(core, ocore)
    assert np.array_equal(labels, ol)
    deg = h.neighbor_counts(torch_mod.from_numpy(pts).cuda(), eps).cpu().numpy()
    assert np.array_equal(deg, odeg)


@pytest.mark.parametrize("seed,rows", [(2, 7), (5, 7), (7, 20), (10, 7), (57, 20)])
def test_batch_partition_changes_border_labels_exactly_like_reference(h, torch_mod, seed, rows):
    """Cases where RAFT's batch-local weak-CC + merge gives an ambiguous border a different
    cluster than the one-batch run; the GPU must reproduce the batched answer."""
    rng = np.random.default_rng(seed)
    pts = rng.uniform(0, 3, size=(60, 2)).astype(np.float32)
    eps, ms = [0.35, 0.5], [3, 5]
    budget = dm.max_bytes_for_batch_size(60, 2, 2, rows, "cuvs", 0, "int32")
    labels, _, r = gpu_fit(h, torch_mod, pts, eps, ms, max_bytes_per_batch=budget, index="int32")
    assert r.stats["batch_size"] == rows
    ol, _, _ = oracle.fit_multi(pts, eps, ms, rows)
    one, _, _ = oracle.fit_multi(pts, eps, ms)
    assert not np.array_equal(ol, one)  # the case really is batch dependent
    assert np.array_equal(labels, ol)


def test_determinism_three_runs(h, torch_mod):
    rng = np.random.default_rng(77)
    pts = blobs(rng, 20000, 8, centers=30, spread=0.8, noise_frac=0.05, box=10.0)
    eps, ms = [0.6, 0.9, 1.2], [5, 10]
    budget = dm.max_bytes_for_batch_size(20000, 3, 2, 3000, "cuvs")
    runs = [gpu_fit(h, torch_mod, pts, eps, ms, max_bytes_per_batch=budget)[0] for _ in range(3)]
    assert all(np.array_equal(runs[0], x) for x in runs[1:])
    ol, _, _ = oracle.fit_multi(pts, eps, ms, 3000)
    assert np.array_equal(runs[0], ol)


def test_edge_cases(h, torch_mod):
    # all duplicates, eps^2 underflowing to zero, huge coordinates whose squares overflow
    dup = np.zeros((300, 3), dtype=np.float32)
    lab, core, _ = gpu_fit(h, torch_mod, dup, [1e-30, 1.0], [1, 300, 301])
    ol, oc, _ = oracle.fit_multi(dup, [1e-30, 1.0], [1, 300, 301])
    assert np.array_equal(lab, ol) and np.array_equal(core, oc)
    big = np.asarray([[0.0], [3e38], [-3e38], [3e38]], dtype=np.float32)
    lab, _, _ = gpu_fit(h, torch_mod, big, [1.0], [2])
    ol, _, _ = oracle.fit_multi(big, [1.0], [2])
    assert np.array_equal(lab, ol)


def test_errors(h, torch_mod):
    x = np.ones((10, 2), dtype=np.float32)
    x[3, 1] = np.nan
    with pytest.raises(dm.DbmError) as ei:
        h.fit_multi(torch_mod.from_numpy(x).cuda(), [0.5], [2])
    assert ei.value.code == -10
    with pytest.raises(dm.DbmError) as ei:
        h.fit_multi(torch_mod.ones((1000, 2), device="cuda"), [0.5], [2], max_bytes_per_batch=100)
    assert ei.value.code == -2
    # the handle stays usable after errors
    lab, _, _ = gpu_fit(h, torch_mod, np.zeros((5, 2), np.float32), [0.1], [2])
    assert lab.tolist() == [[0] * 5]


def test_workspace_reused_across_calls(h, torch_mod):
    rng = np.random.default_rng(5)
    pts = blobs(rng, 5000, 4, centers=5, spread=0.5, noise_frac=0.1, box=5.0)
    gpu_fit(h, torch_mod, pts, [0.5, 0.8], [4])
    before = h.workspace_bytes
    gpu_fit(h, torch_mod, pts, [0.5, 0.8], [4])
    assert h.workspace_bytes == before


def sampled_checks(h, torch, pts, eps, ms, sample, **kw):
    """Size-independent checks at full size: exact degrees of sampled rows against the
    oracle, core masks from them, and the DBSCAN structure of the labels around them."""
    x = torch.from_numpy(pts).cuda()
    r = h.fit_multi(x, eps, ms, return_core=True, **kw)
    labels = r.labels.cpu().numpy()
    core = r.core.cpu().numpy().astype(bool)
    deg = h.neighbor_counts(x, eps).cpu().numpy()
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(len(pts), size=sample, replace=False))
    k, l = len(eps), len(ms)
    for r0 in rows:
        codes, odeg = oracle.codes_degrees(pts, eps, row0=int(r0), rows=1)
        assert np.array_equal(deg[:, r0], odeg[:, 0])
        for e in range(k):
            nbrs = np.flatnonzero(codes[0] <= e)
            for m in range(l):
                cfg = e * l + m
                assert core[cfg, r0] == (odeg[e, 0] >= ms[m])
                lab = labels[cfg]
                core_nbrs = nbrs[core[cfg, nbrs]]
                if core[cfg, r0]:
                    assert np.all(lab[core_nbrs] == lab[r0])
                elif core_nbrs.size == 0:
                    assert lab[r0] == -1
                else:
                    assert lab[r0] in set(lab[core_nbrs].tolist())
    for cfg in range(k * l):
        lab = labels[cfg]
        ids = lab[lab >= 0]
        if ids.size:
            # ids are 0..C-1, ordered by each cluster's smallest core index
            assert ids.max() + 1 == np.unique(ids).size
            cl = lab[core[cfg]]
            idx = np.flatnonzero(core[cfg])
            firsts = np.full(ids.max() + 1, -1)
            seen = np.zeros(ids.max() + 1, dtype=bool)
            order = np.unique(cl, return_index=True)
            firsts[order[0]] = idx[order[1]]
            assert np.all(np.diff(firsts) > 0)
    return r


def test_multi_eps_full_size_properties(h, torch_mod):
    """BASELINE Multi-EPS shape: N=100,000, D=8, k=5, l=1."""
    rng = np.random.default_rng(0)
    n = 100_000
    c = rng.uniform(-10, 10, size=(20, 8))
    m = n - n // 20
    sd = rng.uniform(0.5, 1.0, size=20)
    a = rng.integers(0, 20, size=m)
    pts = np.vstack([c[a] + rng.normal(size=(m, 8)) * sd[a, None],
                     rng.uniform(-10, 10, size=(n - m, 8))]).astype(np.float32)
    r = sampled_checks(h, torch_mod, pts, [0.4, 0.6, 0.8, 1.0, 1.2], [10], 48)
    assert r.stats["batches"] >= 1


def test_multi_both_large_properties(h, torch_mod):
    """BASELINE Multi-Both shape: N=1,000,000, D=33 (last column zero), 4x4 grid, >= 4 batches."""
    rng = np.random.default_rng(0)
    n = 1_000_000
    c = rng.uniform(-20, 20, size=(100, 32))
    m = n - n // 20
    sd = rng.uniform(0.8, 1.5, size=100)
    a = rng.integers(0, 100, size=m)
    pts = np.zeros((n, 33), dtype=np.float32)
    pts[:m, :32] = c[a] + rng.normal(size=(m, 32)) * sd[a, None]
    pts[m:, :32] = rng.uniform(-20, 20, size=(n - m, 32))
    budget = dm.max_bytes_for_batch_size(n, 4, 4, n // 4, "cuvs", 64)
    r = sampled_checks(h, torch_mod, pts, [3.0, 3.5, 4.0, 4.5], [5, 10, 20, 40], 16,
                       max_bytes_per_batch=budget, neigh_per_row=64)
    assert r.stats["batches"] >= 4


@pytest.mark.parametrize("route", ["annotated", "dense"])
@pytest.mark.parametrize("rows", [None, 1500, 400])
def test_routes_and_batches_match_oracle_on_medium_case(h, torch_mod, route, rows):
    """Both routes (compacted per-eps slabs vs eps read from the max-eps codes) with one and
    several batches, on a case dense enough that every eps has many edges."""
    rng = np.random.default_rng(321)
    n = 6000
    pts = blobs(rng, n, 5, centers=8, spread=0.6, noise_frac=0.08, box=4.0)
    eps, ms = [0.45, 0.6, 0.8, 1.0], [3, 8, 20]
    kw = dict(route=route, index="int32")
    if rows:
        kw["max_bytes_per_batch"] = dm.max_bytes_for_batch_size(n, 4, 3, rows, "cuvs", 0, "int32")
    labels, core, r = gpu_fit(h, torch_mod, pts, eps, ms, **kw)
    assert set(r.batch_routes) == {route}
    ol, oc, _ = oracle.fit_multi(pts, eps, ms, r.stats["batch_size"])
    assert np.array_equal(labels, ol) and np.array_equal(core, oc)


def test_config_range_fit_from_graph_matches_full_fit(h, torch_mod):
    """dbm_distance_shard over all shards + dbm_fit_multi_from_graph on config sub-ranges gives
    the rows of the full fit (the multi-GPU building blocks, exercised on one GPU)."""
    from dbscan_multi import parallel

    rng = np.random.default_rng(99)
    pts = blobs(rng, 9000, 6, centers=12, spread=0.7, noise_frac=0.05, box=6.0)
    x = torch_mod.from_numpy(pts).cuda()
    eps, ms = [0.6, 0.9, 1.2], [4, 9]
    budget = dm.max_bytes_for_batch_size(9000, 3, 2, 2500, "cuvs")
    full = h.fit_multi(x, eps, ms, max_bytes_per_batch=budget).labels.cpu().numpy()
    st = parallel.DeviceStages(h)
    e = dm.normalize_eps(eps)
    m = dm.normalize_min_samples(ms)
    hists, parts = [], []
    for shard in range(3):
        hh, ee = st.distance_shard(x, e, shard, 3, 1024)
        hists.append(hh.clone())
        parts.append(ee.clone())
    hist = sum(hists)
    edges = torch_mod.cat(parts)
    opt = dm.Options(0, 0, 0, 0, budget, 0)
    for c0, c1 in [(0, 2), (2, 5), (5, 6), (0, 6)]:
        lab, stats, _ = st.fit_from_graph(9000, 6, e, m, hist, edges, c0, c1, opt)
        assert np.array_equal(lab[c0:c1].cpu().numpy(), full[c0:c1])


def test_core_sample_indices_follow_the_core_masks(h, torch_mod):
    """sklearn/cuML core_sample_indices_ per labelling: ascending core indices, then -1
    (third_party/cuml/cpp/src/dbscan/runner.cuh:406-430), from the fit's core masks."""
    name = CASES[3]
    pts, eps, ms, _ = load_case(name)
    _, core, _ = gpu_fit(h, torch_mod, pts, eps, ms)
    got = h.core_sample_indices(core.astype(np.uint8))
    assert got.shape == core.shape and got.dtype == np.int32
    for c in range(core.shape[0]):
        idx = np.flatnonzero(core[c]).astype(np.int32)
        assert np.array_equal(got[c, : len(idx)], idx)
        assert (got[c, len(idx):] == -1).all()
    x = torch_mod.from_numpy(np.ascontiguousarray(pts, dtype=np.float32)).cuda()
    r = h.fit_multi(x, eps, ms, return_core=True)
    dev = h.core_sample_indices(r.core)
    assert dev.is_cuda and np.array_equal(dev.cpu().numpy(), got)


@pytest.mark.parametrize("route,rows", [("auto", None), ("dense", 700), ("annotated", 2000)])
def test_dense_stress_calibrated_grid_matches_oracle(h, torch_mod, route, rows):
    """The dense-route stress shape (D = 64, 10 blobs of std 2 in [-5,5]^64, no noise, minPts
    {10, 50, 200}) with eps at the 5/10/20% quantiles of sampled pair distances, as the bench's
    calibrated workload sets them: the largest eps links ~20% of all pairs, most tile pairs
    overflow the screen's candidate queue and go to the exact kernel, and the core graph has
    giant components."""
    import bench

    cfg = dict(bench.CONFIGS["c5q"], n=5000)  # >= 4096: the screened pass runs
    pts = bench.make_points(cfg, 3)
    eps = bench.workload_eps(cfg, pts)
    ms = cfg["min_samples"]
    kw = dict(index="int32")
    if route != "auto":
        kw["route"] = route
    if rows:
        kw["max_bytes_per_batch"] = dm.max_bytes_for_batch_size(len(pts), len(eps), len(ms), rows, "cuvs", 0,
                                                                "int32")
    labels, core, r = gpu_fit(h, torch_mod, pts, eps, ms, **kw)
    assert r.stats["screened_tile_pairs"] > 0 and r.stats["fallback_tile_pairs"] > 0
    ol, oc, odeg = oracle.fit_multi(pts, eps, ms, r.stats["batch_size"])
    assert np.array_equal(core, oc)
    assert np.array_equal(labels, ol)
    assert (odeg[-1] - 1).sum() > 0.15 * len(pts) * (len(pts) - 1)  # really dense
