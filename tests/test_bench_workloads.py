"""The bench's workload definitions (no GPU): the calibrated dense-stress eps really sit at the
requested pair-distance quantiles, deterministically."""

from __future__ import annotations

import numpy as np

import bench


def test_calibrated_eps_hit_their_quantiles_and_are_deterministic():
    cfg = dict(bench.CONFIGS["c5q"], n=20_000)
    pts = bench.make_points(cfg, 0)
    eps = bench.workload_eps(cfg, pts)
    assert eps == bench.workload_eps(cfg, pts)
    assert eps == sorted(eps) and len(eps) == 3
    assert all(float(np.float32(e)) == e for e in eps)
    rng = np.random.default_rng(11)
    i = rng.integers(0, len(pts), 50_000)
    j = (i + rng.integers(1, len(pts), 50_000)) % len(pts)
    dist = np.sqrt(((pts[i].astype(np.float64) - pts[j]) ** 2).sum(axis=1))
    for e, q in zip(eps, cfg["eps_quantiles"]):
        assert abs((dist <= e).mean() - q) < 0.01


def test_fixed_eps_workloads_keep_their_grid():
    for name, cfg in bench.CONFIGS.items():
        if cfg.get("eps"):
            assert bench.workload_eps(cfg, np.zeros((4, cfg["d"]), np.float32)) == list(cfg["eps"])


def test_labelling_roofline_counts_compaction_only_where_the_fit_compacts():
    """The labelling's algorithmic bytes: one CC sweep per configuration, plus the smaller-eps
    compaction only for dense graphs routed annotated (sparse batches read each entry's eps from
    its code and compact nothing)."""
    n, l = 1000, 2
    stats = {"annotated_batches": 3}
    sparse = [4 * n, 8 * n, 16 * n]
    dense = [100 * n, 200 * n, 400 * n]
    cc = lambda nnz: sum(l * (8.0 * v + 8.0 * n + n / 8.0) for v in nnz)
    r = bench.label_roofline(sparse, n, l, stats, [1.0], 1)
    assert r["bytes_per_grid"] == cc(sparse)
    r = bench.label_roofline(dense, n, l, stats, [1.0], 1)
    assert r["bytes_per_grid"] == cc(dense) + 4.0 * dense[-1] + 8.0 * sum(dense[:-1])
    r = bench.label_roofline(dense, n, l, {"annotated_batches": 0}, [1.0], 1)
    assert r["bytes_per_grid"] == cc(dense)
