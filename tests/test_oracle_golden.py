"""Pins the CPU oracle against the reference's own golden vectors and known answers.

The oracle (oracle/dbm_oracle.c) is the checker for every GPU parity test, so it is first
checked here against:
  * the 13 golden label bundles the reference ships (every mode of the reference binary,
    raw-equal per case), unbatched and with the batch sizes of the reference's 1 MB
    "batched" modes (cuVS 98 rows, codes 164 rows for forced_batches_2d);
  * the reference selftest's recorded answers (clusters and noise per configuration, and
    4 batches of 750 rows giving the same labels).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import batching
import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("0*.npz"))


def load_case(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return z["points"], z["eps"].astype(np.float32), z["min_samples"].astype(np.int32), z["labels"]


def test_thirteen_cases_present():
    assert len(CASES) == 13


@pytest.mark.parametrize("name", CASES)
def test_oracle_raw_equal_to_reference_labels(name):
    pts, eps, ms, expected = load_case(name)
    labels, core, deg = oracle.fit_multi(pts, eps, ms)
    assert np.array_equal(labels, expected)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("use_cuvs", [True, False])
def test_oracle_batched_modes_match_reference(name, use_cuvs):
    pts, eps, ms, expected = load_case(name)
    n, k, l = len(pts), len(eps), len(ms)
    bs = batching.compute_batch_size(n, k, l, 1_000_000, use_cuvs, 0, 32)
    labels, _, _ = oracle.fit_multi(pts, eps, ms, bs)
    assert np.array_equal(labels, expected)


def test_forced_batches_case_really_batches():
    pts, eps, ms, _ = load_case("009_forced_batches_2d")
    n = len(pts)
    assert batching.compute_batch_size(n, 2, 2, 1_000_000, True) == 98
    assert batching.compute_batch_size(n, 2, 2, 1_000_000, False) == 164


def test_selftest_known_answers():
    spec = json.loads((GOLDEN / "selftest_answers.json").read_text())
    pts = oracle.selftest_points(1000, 2, 42)
    labels, _, _ = oracle.fit_multi(pts, spec["eps"], spec["min_samples"])
    for cfg, ans in enumerate(spec["configurations"]):
        lab = labels[cfg]
        assert int(lab.max()) + 1 == ans["clusters"]
        assert int((lab < 0).sum()) == ans["noise"]
    # forced batching: the reference used a budget that yields 4 x 750 rows
    budget = batching.max_bytes_for_batch_size(3000, 3, 3, 750, True)
    bs = batching.compute_batch_size(3000, 3, 3, budget, True)
    assert bs == spec["forced_batch_size"] == 750
    batched, _, _ = oracle.fit_multi(pts, spec["eps"], spec["min_samples"], bs)
    assert np.array_equal(batched, labels)


@pytest.mark.parametrize("d", [2, 8, 16, 32, 33])
def test_selftest_three_clusters_every_dimension(d):
    pts = oracle.selftest_points(500, d, 42)
    for eps in ([0.8], [0.3, 0.5, 0.8], [0.2, 0.3, 0.5, 0.65, 0.8]):
        labels, _, _ = oracle.fit_multi(pts, eps, [4])
        assert int(labels[-1].max()) + 1 == 3


def test_closed_ball_boundary():
    pts = np.asarray([[0.0], [1.0]], dtype=np.float32)
    labels, core, deg = oracle.fit_multi(pts, [1.0], [2])
    assert deg.tolist() == [[2, 2]] and labels.tolist() == [[0, 0]]
    out = np.nextafter(np.float32(1.0), np.float32(2.0))
    pts2 = np.asarray([[0.0], [out]], dtype=np.float32)
    labels, core, deg = oracle.fit_multi(pts2, [1.0], [2])
    assert deg.tolist() == [[1, 1]] and labels.tolist() == [[-1, -1]]


def test_sequential_fma_rounding_is_what_is_restated():
    # a pair whose squared distance differs between fma-chain and separately-rounded sums
    rng = np.random.default_rng(7)
    x = rng.normal(size=(2, 33)).astype(np.float32)
    acc = np.float32(0)
    for t in range(33):
        diff = np.float32(x[0, t] - x[1, t])
        acc = np.float32(np.float64(diff) * np.float64(diff) + np.float64(acc))  # exact fma for f32
    eps = np.float32(np.sqrt(np.float64(acc)))
    while np.float32(eps * eps) < acc:
        eps = np.nextafter(eps, np.float32(np.inf))
    codes, deg = oracle.codes_degrees(x, [eps])
    assert codes[0, 1] == 0 and deg[0].tolist() == [2, 2]
    below = np.nextafter(eps, np.float32(0))
    while np.float32(below * below) >= acc:
        below = np.nextafter(below, np.float32(0))
    codes, deg = oracle.codes_degrees(x, [below])
    assert codes[0, 1] == 255


def test_route_rule():
    # annotate iff nnz*D*40 < (k-1)*(pairs*D + 6e10)
    assert oracle.annotate_pays(4_000_000, 4000 * 4000, 5, 2)
    assert not oracle.annotate_pays(1_170_000_000, 64000 * 64000, 5, 64)
