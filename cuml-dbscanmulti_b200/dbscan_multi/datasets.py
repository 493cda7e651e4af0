"""The reference's on-disk dataset format: ``<base>.f32`` + ``<base>.labels.i32`` + ``<base>.json``.

Written by the reference's generator (tools/gerar_datasets.py:648-706) and read by its tools
(tools/bench_vs_cuml.py ``--meta``): float32 points, row-major, no header; int32 ground-truth
labels; a JSON document with the shape, the grid (``eps`` and ``min_samples`` already sorted,
eps-major configuration order), the protocol tag and SHA-256 digests of the files.

``load_dataset(meta_path)`` checks what the reference's tools check before a run (protocol,
dtype, layout, sizes, digests; optionally the dataset name, N, the eps count and the eps
quantiles, as tools/gerar_datasets.py:617-645 does) and returns the points and the grid,
ready for ``fit_multi(points, ds.eps, ds.min_samples)``; ``write_dataset`` writes the same
layout, and ``normalize_minmax`` is the generator's per-column scaling (:131-138).
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Sequence

import numpy as np

PROTOCOL = "knn-sample-rank-v2"


class DatasetError(ValueError):
    pass


@dataclass
class Dataset:
    points: np.ndarray          # (n, d) float32
    eps: list[float]
    min_samples: list[int]
    labels_true: np.ndarray | None
    meta: dict[str, Any] = field(default_factory=dict)

    @property
    def n(self) -> int:
        return int(self.points.shape[0])

    @property
    def d(self) -> int:
        return int(self.points.shape[1])


def sha256_file(path: Path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def normalize_minmax(x: np.ndarray) -> np.ndarray:
    """Each column scaled to [0, 1] in float32; a constant column keeps span 1 (becomes 0)."""
    x = np.asarray(x, dtype=np.float32)
    lo = x.min(axis=0)
    span = x.max(axis=0) - lo
    span[span == 0.0] = 1.0
    return ((x - lo) / span).astype(np.float32)


def load_dataset(meta_path: str | Path, *, verify: bool = True, require_protocol: bool = True,
                 dataset: str | None = None, n: int | None = None, eps_count: int | None = None,
                 eps_quantiles: Sequence[float] | None = None) -> Dataset:
    meta_path = Path(meta_path)
    meta = json.loads(meta_path.read_text(encoding="utf-8"))
    if require_protocol and meta.get("protocolo_dataset") != PROTOCOL:
        raise DatasetError(f"{meta_path}: dataset protocol {meta.get('protocolo_dataset')!r}, expected {PROTOCOL!r}")
    if dataset is not None and meta.get("dataset") != dataset:
        raise DatasetError(f"{meta_path}: dataset {meta.get('dataset')!r}, expected {dataset!r}")
    if n is not None and meta.get("n") != n:
        raise DatasetError(f"{meta_path}: N {meta.get('n')!r}, expected {n}")
    if eps_count is not None and len(meta.get("eps", [])) != eps_count:
        raise DatasetError(f"{meta_path}: {len(meta.get('eps', []))} eps values, expected {eps_count}")
    if eps_quantiles is not None and tuple(map(float, meta.get("quantis_eps", []))) != tuple(map(float, eps_quantiles)):
        raise DatasetError(f"{meta_path}: eps quantiles {meta.get('quantis_eps')!r}, expected {list(eps_quantiles)!r}")
    if meta.get("dtype", "float32") != "float32" or meta.get("layout", "row-major") != "row-major":
        raise DatasetError(f"{meta_path}: only float32 row-major points are supported")
    n, d = int(meta["n"]), int(meta["d"])
    files = meta.get("arquivos", {})
    points_path = meta_path.parent / files.get("points", meta_path.with_suffix(".f32").name)
    if not points_path.exists():
        raise DatasetError(f"points file {points_path} is missing")
    if points_path.stat().st_size != n * d * 4:
        raise DatasetError(f"{points_path} has {points_path.stat().st_size} bytes, expected {n * d * 4}")
    digests = meta.get("sha256", {})
    if verify and "points" in digests and sha256_file(points_path) != digests["points"]:
        raise DatasetError(f"{points_path}: SHA-256 does not match the metadata")
    points = np.fromfile(points_path, dtype=np.float32).reshape(n, d)
    labels = None
    lab_name = files.get("labels_verdadeiros")
    if lab_name:
        lab_path = meta_path.parent / lab_name
        if lab_path.exists():
            if verify and "labels_verdadeiros" in digests and sha256_file(lab_path) != digests["labels_verdadeiros"]:
                raise DatasetError(f"{lab_path}: SHA-256 does not match the metadata")
            labels = np.fromfile(lab_path, dtype=np.int32)
            if labels.size != n:
                raise DatasetError(f"{lab_path} holds {labels.size} labels, expected {n}")
    eps = [float(v) for v in meta["eps"]]
    min_samples = [int(v) for v in meta["min_samples"]]
    if eps != sorted(set(eps)) or min_samples != sorted(set(min_samples)):
        raise DatasetError(f"{meta_path}: the grid must be sorted and without duplicates")
    if meta.get("config_order", "eps_major") != "eps_major":
        raise DatasetError(f"{meta_path}: only eps-major configuration order is defined")
    return Dataset(points=points, eps=eps, min_samples=min_samples, labels_true=labels, meta=meta)


def write_dataset(base: str | Path, points: np.ndarray, eps: Sequence[float], min_samples: Sequence[int],
                  labels_true: np.ndarray | None = None, name: str | None = None,
                  extra: dict[str, Any] | None = None) -> Path:
    """Writes ``<base>.f32``, optionally ``<base>.labels.i32``, and ``<base>.json``."""
    base = Path(base)
    base.parent.mkdir(parents=True, exist_ok=True)
    x = np.ascontiguousarray(points, dtype=np.float32)
    if x.ndim != 2:
        raise DatasetError("points must be (n, d)")
    e = sorted({float(v) for v in eps})
    m = sorted({int(v) for v in min_samples})
    pts_path = base.with_name(base.name + ".f32")
    x.tofile(pts_path)
    files = {"points": pts_path.name}
    digests = {"points": sha256_file(pts_path)}
    if labels_true is not None:
        lab_path = base.with_name(base.name + ".labels.i32")
        np.ascontiguousarray(labels_true, dtype=np.int32).tofile(lab_path)
        files["labels_verdadeiros"] = lab_path.name
        digests["labels_verdadeiros"] = sha256_file(lab_path)
    meta = {
        "protocolo_dataset": PROTOCOL,
        "dataset": name or base.name,
        "n": int(x.shape[0]),
        "d": int(x.shape[1]),
        "dtype": "float32",
        "layout": "row-major",
        "eps": e,
        "min_samples": m,
        "configuration_count": len(e) * len(m),
        "config_order": "eps_major",
        "arquivos": files,
        "sha256": digests,
    }
    if extra:
        meta.update(extra)
    meta_path = base.with_name(base.name + ".json")
    meta_path.write_text(json.dumps(meta, indent=2, ensure_ascii=False), encoding="utf-8")
    return meta_path


# ---- grid heuristics: which (eps, minPts) grid to run on a dataset ------------------------------
# The reference's generator proposes a grid per dataset (tools/gerar_datasets.py:493-605); these
# functions restate its rules so a grid can be chosen without it: minPts from an intrinsic
# dimension estimate and log2(N), eps from quantiles of a sampled k-distance curve (the automated
# form of the classic k-distance plot).  Same samples, same neighbour searches, same arithmetic,
# so the same grid (pinned against outputs of the reference generator in tests/test_datasets.py).

GRID_SEED = 42  # the generator's default seed: samples drawn with it select the same rows


@dataclass
class GridSuggestion:
    eps: list[float]
    min_samples: list[int]
    min_samples_reference: int   # the minPts whose k-distance curve gave the eps values
    intrinsic_dimension: float
    sample_rank: int             # neighbour rank used in the sample (corrected for its size)


def _sample_rows(n: int, max_points: int, seed: int) -> np.ndarray:
    """Indices of a uniform sample without replacement (all rows when n <= max_points)."""
    if n <= int(max_points):
        return np.arange(n)
    return np.random.default_rng(seed).choice(n, size=int(max_points), replace=False)


def _neighbour_distances(x: np.ndarray, k: int) -> np.ndarray:
    from sklearn.neighbors import NearestNeighbors

    return NearestNeighbors(n_neighbors=int(k), algorithm="auto").fit(x).kneighbors(x)[0]


def intrinsic_dimension(x, k: int = 20, sample_size: int = 5000, seed: int = GRID_SEED) -> float:
    """Levina-Bickel maximum-likelihood estimate of the intrinsic dimension (median over a
    sample of the per-point estimates from the k nearest neighbours), clipped to [1, 2D].
    A curve or a ring in many dimensions comes out near 1, which is what minPts should follow."""
    x = np.asarray(x, dtype=np.float32)
    xs = np.ascontiguousarray(x[_sample_rows(x.shape[0], sample_size, seed)], dtype=np.float32)
    kk = int(min(max(4, k), xs.shape[0] - 1))
    if kk < 3:
        return float(x.shape[1])
    dist = _neighbour_distances(xs, kk + 1)[:, 1:]  # drop each point itself (distance 0)
    tiny = 1e-12
    inv = np.mean(np.log((dist[:, -1:] + tiny) / (dist[:, :-1] + tiny)), axis=1)
    local = 1.0 / np.maximum(inv, tiny)
    return float(np.clip(float(np.nanmedian(local)), 1.0, max(1.0, 2.0 * x.shape[1])))


def suggest_min_samples(x, sample_size: int = 5000, max_min_samples: int = 256,
                        seed: int = GRID_SEED) -> tuple[list[int], float]:
    """minPts candidates {b/2, b, 2b, 4b} clipped to [4, max], with b = max(4, ceil(2 dim),
    ceil(log2 N)); returns them ascending with the dimension estimate."""
    x = np.asarray(x, dtype=np.float32)
    dim = intrinsic_dimension(x, sample_size=sample_size, seed=seed)
    base = max(4, int(np.ceil(2.0 * dim)), int(np.ceil(np.log2(max(x.shape[0], 2)))))
    cands = sorted({int(np.clip(c, 4, max_min_samples)) for c in (base // 2, base, 2 * base, 4 * base)})
    return cands, dim


def suggest_eps(x, min_samples: int, quantiles=(0.50, 0.70, 0.85), max_points: int = 60000,
                seed: int = GRID_SEED, labels=None) -> tuple[list[float], int]:
    """eps candidates at `quantiles` of the k-distance curve of a sample of at most max_points
    rows (k = min_samples, the point itself included).  A sample of s of N rows uses the rank
    1 + round((min_samples - 1)(s - 1)/(N - 1)), the rank whose distance in the sample estimates
    the full data's min_samples-th neighbour.  With true labels given, noise rows (label < 0)
    stay in the neighbour index but their own k-distances are left out of the quantiles when
    enough rows remain (the uniform noise tail would otherwise pull the largest eps far beyond
    the clusters).  Returns the distinct float32 values ascending and the rank used."""
    x = np.asarray(x, dtype=np.float32)
    idx = _sample_rows(x.shape[0], max_points, seed)
    xs = x[idx]
    if x.shape[0] <= 1 or xs.shape[0] <= 1:
        k = 1
    else:
        frac = (xs.shape[0] - 1) / (x.shape[0] - 1)
        k = int(np.clip(1 + int(round(max(0, int(min_samples) - 1) * frac)), 2, xs.shape[0]))
    kth = _neighbour_distances(xs, k)[:, -1]
    if labels is not None:
        structured = np.asarray(labels)[idx] >= 0
        if structured.sum() >= max(50, 0.1 * kth.size):
            kth = kth[structured]
    kth = np.sort(kth)
    eps = np.asarray([np.quantile(kth, q) for q in quantiles], dtype=np.float32)
    eps = np.unique(np.maximum(eps, np.float32(1e-6))).astype(np.float32)
    return [float(v) for v in eps], int(k)


def suggest_grid(x, quantiles=(0.50, 0.70, 0.85), seed: int = GRID_SEED, labels=None) -> GridSuggestion:
    """The full grid: the minPts candidates, and eps from the k-distance curve of the middle
    candidate (3 x 4 = 12 configurations with the default quantiles)."""
    ms, dim = suggest_min_samples(x, seed=seed)
    ref = ms[len(ms) // 2]
    eps, k = suggest_eps(x, ref, quantiles=quantiles, seed=seed, labels=labels)
    return GridSuggestion(eps=eps, min_samples=ms, min_samples_reference=ref, intrinsic_dimension=dim,
                          sample_rank=k)
