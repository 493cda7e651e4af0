"""The memory-bounded fit (the graph built one row batch at a time, dbm_set_graph_mode) against the
reference's goldens, the oracle and the one-shot fit.

The reference bounds its memory by its budget: pass 2 rebuilds each batch's CSR into buffers
sized by the largest batch (runner_multi.cuh:1020-1041, 1100-1226).  Here the streamed fit
re-orders the points batch-major, re-derives each batch's neighbour pairs from the tile pairs
touching the batch and builds that batch's CSR rows only; the labels must not change in any mode:
every golden bundle in every mode of the reference binary, seeded batched cases on both routes,
the exact-kernel regime (N < 4096, D > 64) and the screened regime, and the automatic switch when
the whole graph does not fit the budget.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import dbscan_multi as dm
import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("0*.npz"))

MODES = {
    "cuvs_auto_i32": dict(backend="cuvs", index="int32"),
    "cuvs_annotated_i32": dict(backend="cuvs", index="int32", route="annotated"),
    "cuvs_dense_i32": dict(backend="cuvs", index="int32", route="dense"),
    "codes_i64": dict(backend="codes", index="int64"),
    "cuvs_batched": dict(backend="cuvs", index="int32", max_bytes_per_batch=1_000_000),
    "codes_batched": dict(backend="codes", index="int32", max_bytes_per_batch=1_000_000),
}


@pytest.fixture(scope="module")
def torch_mod():
    import torch

    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def streamed(torch_mod):
    h = dm.DbscanMulti(0)
    h.set_graph_mode("streamed")
    yield h
    h.close()


@pytest.fixture(scope="module")
def oneshot(torch_mod):
    h = dm.DbscanMulti(0)
    h.set_graph_mode("oneshot")
    yield h
    h.close()


def fit(h, torch, pts, eps, ms, **kw):
    x = torch.from_numpy(np.ascontiguousarray(pts, dtype=np.float32)).to("cuda:0")
    r = h.fit_multi(x, eps, ms, return_core=True, **kw)
    return r.labels.cpu().numpy(), r.core.cpu().numpy().astype(bool), r


@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("name", CASES)
def test_golden_bundles_streamed(streamed, torch_mod, name, mode):
    z = np.load(GOLDEN / f"{name}.npz")
    labels, _, r = fit(streamed, torch_mod, z["points"], z["eps"].astype(np.float32),
                       z["min_samples"].astype(np.int32), **MODES[mode])
    assert r.stats["streamed"] == 1
    assert np.array_equal(labels, z["labels"]), f"{name}/{mode}"


def blobs(seed, n, d, centers, std, noise, box):
    rng = np.random.default_rng(seed)
    c = rng.uniform(-box, box, size=(centers, d))
    m = n - int(noise * n)
    pts = np.vstack([c[rng.integers(0, centers, m)] + rng.normal(0, std, (m, d)),
                     rng.uniform(-box, box, (n - m, d))]).astype(np.float32)
    return pts


RANDOM = {
    # name: (points, eps, min_samples, rows per batch)
    "d3_dense_small": (blobs(11, 3000, 3, 4, 0.5, 0.05, 4), [0.3, 0.5, 0.8], [4, 12, 30], 431),
    "d8_sparse_screened": (blobs(12, 12000, 8, 10, 0.6, 0.05, 8), [0.5, 0.8, 1.1], [5, 10], 1700),
    "d33_c4_like": (np.hstack([blobs(13, 9000, 32, 12, 1.1, 0.05, 20), np.zeros((9000, 1), np.float32)]),
                    [3.0, 3.5, 4.0, 4.5], [5, 10, 20, 40], 2048),
    "d72_exact_only": (blobs(14, 5000, 72, 6, 1.5, 0.05, 6), [9.0, 11.0], [3, 9], 777),
    "k1_one_eps": (blobs(15, 6000, 2, 6, 0.3, 0.1, 5), [0.12], [3, 6, 20], 600),
}


@pytest.mark.parametrize("route", ["annotated", "dense"])
@pytest.mark.parametrize("name", sorted(RANDOM))
def test_streamed_equals_oneshot_and_oracle(streamed, oneshot, torch_mod, name, route):
    pts, eps, ms, rows = RANDOM[name]
    n = len(pts)
    budget = dm.max_bytes_for_batch_size(n, len(eps), len(ms), rows, "cuvs")
    kw = dict(max_bytes_per_batch=budget, route=route if len(eps) > 1 else "auto")
    lab_s, core_s, r_s = fit(streamed, torch_mod, pts, eps, ms, **kw)
    lab_o, core_o, r_o = fit(oneshot, torch_mod, pts, eps, ms, **kw)
    assert r_s.stats["streamed"] == 1 and r_o.stats["streamed"] == 0
    assert r_s.stats["batch_size"] == rows == r_o.stats["batch_size"]
    want, want_core, _ = oracle.fit_multi(pts, eps, ms, rows)
    assert np.array_equal(lab_s, want) and np.array_equal(core_s, want_core)
    assert np.array_equal(lab_o, want)
    assert r_s.batch_routes == r_o.batch_routes


def test_auto_streams_when_the_graph_exceeds_the_budget(torch_mod):
    """A dense graph (~560 neighbours per point) and a budget sized by the reference's rule for
    2,000-row batches with an expected 16 neighbours per row (40 MB): the whole pair list and CSR
    would take 135 MB, more than the budget allows, so the fit builds the graph per batch -- and
    the handle's workspace stays below what the one-shot fit of the same grid holds."""
    pts = blobs(21, 20000, 4, 6, 0.35, 0.0, 3)
    eps, ms = [0.35, 0.6], [10, 50]
    n = len(pts)
    budget = dm.max_bytes_for_batch_size(n, 2, 2, 2000, "cuvs", neigh_per_row=16)
    want, _, _ = oracle.fit_multi(pts, eps, ms, 2000)
    with dm.DbscanMulti(0) as h:
        lab, _, r = fit(h, torch_mod, pts, eps, ms, max_bytes_per_batch=budget, neigh_per_row=16)
        assert r.stats["streamed"] == 1 and r.stats["batches"] == 10
        assert 24 * r.stats["edges"] > 3 * budget
        assert np.array_equal(lab, want)
        ws_streamed = r.stats["workspace_bytes"]
    with dm.DbscanMulti(0) as h:
        h.set_graph_mode("oneshot")
        lab, _, r = fit(h, torch_mod, pts, eps, ms, max_bytes_per_batch=budget, neigh_per_row=16)
        assert r.stats["streamed"] == 0 and np.array_equal(lab, want)
        assert r.stats["workspace_bytes"] > ws_streamed
