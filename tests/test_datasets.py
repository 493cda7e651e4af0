"""The reference's dataset format (points .f32 + labels .i32 + metadata .json)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from dbscan_multi import datasets


def test_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    x = rng.normal(size=(500, 3)).astype(np.float32)
    y = rng.integers(-1, 4, 500).astype(np.int32)
    meta = datasets.write_dataset(tmp_path / "blobs_n500", x, [0.5, 0.2], [10, 5], y)
    ds = datasets.load_dataset(meta)
    assert np.array_equal(ds.points, x) and np.array_equal(ds.labels_true, y)
    assert ds.eps == [pytest.approx(0.2), pytest.approx(0.5)] and ds.min_samples == [5, 10]
    assert ds.meta["configuration_count"] == 4 and ds.meta["config_order"] == "eps_major"


def test_rejects_corruption_and_wrong_protocol(tmp_path):
    x = np.zeros((10, 2), np.float32)
    meta = datasets.write_dataset(tmp_path / "z", x, [0.1], [2])
    pts = tmp_path / "z.f32"
    raw = bytearray(pts.read_bytes())
    raw[0] ^= 1
    pts.write_bytes(bytes(raw))
    with pytest.raises(datasets.DatasetError, match="SHA-256"):
        datasets.load_dataset(meta)
    assert datasets.load_dataset(meta, verify=False).n == 10
    m = json.loads(meta.read_text())
    m["protocolo_dataset"] = "historico"
    meta.write_text(json.dumps(m))
    with pytest.raises(datasets.DatasetError, match="protocol"):
        datasets.load_dataset(meta, verify=False)
    m["protocolo_dataset"] = datasets.PROTOCOL
    m["n"] = 11
    meta.write_text(json.dumps(m))
    with pytest.raises(datasets.DatasetError, match="bytes"):
        datasets.load_dataset(meta, verify=False)


def test_unsorted_grid_is_rejected(tmp_path):
    meta = datasets.write_dataset(tmp_path / "u", np.zeros((4, 1), np.float32), [0.1, 0.2], [2])
    m = json.loads(meta.read_text())
    m["eps"] = [0.2, 0.1]
    meta.write_text(json.dumps(m))
    with pytest.raises(datasets.DatasetError, match="sorted"):
        datasets.load_dataset(meta)


@pytest.mark.gpu
def test_fit_a_written_dataset_through_the_api(tmp_path):
    import dbscan_multi as dm
    import oracle

    rng = np.random.default_rng(5)
    x = np.vstack([rng.normal(c, 0.2, (300, 2)) for c in (0, 2, 4)]).astype(np.float32)
    meta = datasets.write_dataset(tmp_path / "three_n900", x, [0.15, 0.3], [5, 12])
    ds = datasets.load_dataset(meta)
    with dm.DbscanMulti(0) as h:
        r = h.fit_multi(ds.points, ds.eps, ds.min_samples)
    want, _, _ = oracle.fit_multi(ds.points, ds.eps, ds.min_samples)
    assert np.array_equal(r.labels, want)


def test_normalize_minmax():
    x = np.array([[1.0, 5.0, -2.0], [3.0, 5.0, 2.0], [2.0, 5.0, 0.0]], np.float32)
    got = datasets.normalize_minmax(x)
    assert got.dtype == np.float32
    assert np.array_equal(got, np.array([[0, 0, 0], [1, 0, 1], [0.5, 0, 0.5]], np.float32))
    rng = np.random.default_rng(3)
    y = (rng.normal(size=(1000, 4)) * [1, 1e-3, 1e3, 0]).astype(np.float32)
    want = (y - y.min(0)) / np.where(np.ptp(y, 0) == 0, np.float32(1), np.ptp(y, 0))
    assert np.array_equal(datasets.normalize_minmax(y), want.astype(np.float32))


def test_metadata_expectations(tmp_path):
    meta = datasets.write_dataset(tmp_path / "m_n6", np.zeros((6, 2), np.float32), [0.1, 0.2], [3],
                                  name="moons_2d", extra={"quantis_eps": [0.5, 0.7]})
    assert datasets.load_dataset(meta, dataset="moons_2d", n=6, eps_count=2, eps_quantiles=(0.5, 0.7)).n == 6
    for kw, msg in (({"dataset": "rings_2d"}, "dataset"), ({"n": 7}, "N "), ({"eps_count": 3}, "eps values"),
                    ({"eps_quantiles": (0.5, 0.85)}, "quantiles")):
        with pytest.raises(datasets.DatasetError, match=msg):
            datasets.load_dataset(meta, **kw)


def _grid_cases():
    import importlib.util
    import json
    from pathlib import Path

    here = Path(__file__).resolve().parent / "golden"
    spec = importlib.util.spec_from_file_location("grid_fixtures", here / "make_grid_fixtures.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    data = json.loads((here / "grid_heuristics.json").read_text())
    return mod.grid_case_points, data


def test_grid_heuristics_match_the_reference_generator():
    """Each case's points are regenerated from its seed; minPts candidates, the intrinsic
    dimension, the sampled neighbour rank and the eps values (with and without the true labels)
    must equal what the reference generator's heuristics returned for them."""
    from dbscan_multi import datasets as ds

    make, data = _grid_cases()
    assert data["seed"] == ds.GRID_SEED
    for case in data["cases"]:
        x, y = make(case["n"], case["d"], case["centres"], case["std"], case["noise"], case["seed"])
        g = ds.suggest_grid(x, labels=y)
        assert g.min_samples == case["min_samples"], case["name"]
        assert g.min_samples_reference == case["min_samples_reference"]
        assert g.intrinsic_dimension == case["intrinsic_dimension"]
        assert g.sample_rank == case["sample_rank"]
        assert g.eps == case["eps"], case["name"]
        eps_plain, _ = ds.suggest_eps(x, case["min_samples_reference"])
        assert eps_plain == case["eps_without_labels"], case["name"]
