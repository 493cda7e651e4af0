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
