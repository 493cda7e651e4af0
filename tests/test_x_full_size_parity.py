"""Full-size parity: every bench workload (the published configurations C1-C5 and the calibrated
dense C5) at its stated size, through the C ABI, against the oracle.

* C1 (N = 10,000) and C2 (N = 100,000): the whole (k*l, N) label matrix and the core masks are
  compared with the oracle run live (oracle.fit_multi_stream, seconds on the host cores).
* Every workload: the per-configuration SHA-256 of the label rows, and the cluster, noise and
  core counts, against tests/golden/full_size_labels.json, which
  tests/golden/make_full_size_fixtures.py wrote by running the oracle on the same seeded points
  with the same batch partition (C4's 1M points take the oracle ~25 minutes, too long to redo
  here).
The memory budget of each workload is explicit (128 GB) and the batch size must equal the
reference's rule for it, since ambiguous border points follow the batch partition.  This file is
named to run after the faster GPU tests.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import bench
import dbscan_multi as dm
import oracle

pytestmark = pytest.mark.gpu

FIXTURES = json.loads((Path(__file__).resolve().parent / "golden" / "full_size_labels.json").read_text())


@pytest.fixture(scope="module")
def h():
    import torch

    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    handle = dm.DbscanMulti(0)
    yield handle
    handle.close()


def workload(name):
    cfg = dict(bench.CONFIGS[name])
    pts = bench.make_points(cfg, 0)
    eps = bench.workload_eps(cfg, pts)
    return cfg, pts, eps, list(cfg["min_samples"])


def gpu_fit(h, name, return_core=False):
    import torch

    cfg, pts, eps, ms = workload(name)
    x = torch.from_numpy(pts).cuda()
    r = h.fit_multi(x, eps, ms, max_bytes_per_batch=cfg["budget"], neigh_per_row=cfg["npr"],
                    return_core=return_core)
    labels = r.labels.cpu().numpy()
    core = r.core.cpu().numpy().astype(bool) if return_core else None
    del x
    return pts, eps, ms, labels, core, r


def digests(labels):
    return [hashlib.sha256(np.ascontiguousarray(row, dtype="<i4").tobytes()).hexdigest() for row in labels]


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_full_label_matrix_equals_the_oracle(h, name):
    pts, eps, ms, labels, core, r = gpu_fit(h, name, return_core=True)
    fx = FIXTURES[name]
    assert r.stats["batch_size"] == fx["batch_size"] and r.stats["batches"] == fx["batches"]
    want, want_core, _, _ = oracle.fit_multi_stream(pts, eps, ms, r.stats["batch_size"])
    assert np.array_equal(labels, want)
    assert np.array_equal(core, want_core)
    assert digests(labels) == [c["sha256"] for c in fx["configs"]]


@pytest.mark.parametrize("name", ["c3", "c4", "c5", "c5qb", "c5q"])
def test_full_size_labels_match_the_oracle_digests(h, name):
    fx = FIXTURES.get(name)
    assert fx is not None, f"no oracle fixture for {name}"
    if name == "c5qb":
        # a fresh handle: the budget bounds what a fit adds to the handle's workspace, and the
        # shared handle may already hold a one-shot graph from another workload
        with dm.DbscanMulti(0) as fresh:
            pts, eps, ms, labels, _, r = gpu_fit(fresh, name)
    else:
        pts, eps, ms, labels, _, r = gpu_fit(h, name)
    assert hashlib.sha256(pts.tobytes()).hexdigest() == fx["points_sha256"]
    assert [float(e) for e in eps] == fx["eps"] and ms == fx["min_samples"]
    assert r.stats["batch_size"] == fx["batch_size"] and r.stats["batches"] == fx["batches"]
    assert r.stats["total_nnz_max_eps"] == fx["nnz_max_eps"]
    if name == "c5qb":  # 24 bytes per neighbour pair would exceed the budget: per-batch graph
        assert r.stats["streamed"] == 1 and r.stats["workspace_bytes"] < fx["max_bytes_per_batch"]
    got = digests(labels)
    for c, (g, want) in enumerate(zip(got, fx["configs"])):
        row = labels[c]
        assert (int(row.max()) + 1, int((row == -1).sum())) == (want["clusters"], want["noise"]), f"config {c}"
        assert g == want["sha256"], f"config {c}"
