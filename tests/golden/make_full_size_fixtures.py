"""Writes tests/golden/full_size_labels.json: the oracle's labels for every bench workload at its
full size, as per-configuration SHA-256 digests plus cluster, noise and core counts.

The GPU path is compared against these in tests/test_x_full_size_parity.py (and bench.py's
multi-GPU runs compare their labels with a one-GPU fit).  Inputs are exactly the bench's: the
seeded generator `bench.make_points(cfg, seed=0)`, the workload's eps (the calibrated quantiles
for c5q), its minPts and its explicit memory budget; the batch size is the reference's rule for
that budget (oracle/batching.py, runner_multi.cuh:458-499), since ambiguous border points follow
the batch partition.  The oracle runs batch by batch (oracle.fit_multi_stream, only one batch's
neighbour lists in memory) on every host core.

    python tests/golden/make_full_size_fixtures.py [c1 c2 ...]     # default: all workloads

Each workload is written as soon as it finishes (existing entries of other workloads are kept).
Rough cost on 8 cores: c1, c2 seconds; c5 2 min; c3 7 min; c5q, c5qb 5 min; c4 ~25 min.
"""

from __future__ import annotations

import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
for _p in (ROOT, ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import batching  # noqa: E402
import bench  # noqa: E402
import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent / "full_size_labels.json"


def index_bits(n: int) -> int:
    """The reference CLI's --index auto: int64 iff N*N >= INT32_MAX (src/main.cu:681-689)."""
    return 64 if n * n >= 2**31 - 1 else 32


def row_digest(labels_row: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(labels_row, dtype="<i4").tobytes()).hexdigest()


def summarise(labels: np.ndarray, core: np.ndarray) -> list[dict]:
    rows = []
    for c in range(labels.shape[0]):
        lab = labels[c]
        rows.append({"sha256": row_digest(lab), "clusters": int(lab.max()) + 1 if lab.size else 0,
                     "noise": int((lab == -1).sum()), "core": int(core[c].sum())})
    return rows


def workload(name: str) -> dict:
    cfg = dict(bench.CONFIGS[name])
    pts = bench.make_points(cfg, 0)
    eps = bench.workload_eps(cfg, pts)
    ms = list(cfg["min_samples"])
    n, d = pts.shape
    bits = index_bits(n)
    bs = batching.compute_batch_size(n, len(eps), len(ms), cfg["budget"], use_cuvs=True,
                                     neigh_hint=cfg["npr"], index_bits=bits)
    t0 = time.time()
    labels, core, deg, nnz = oracle.fit_multi_stream(pts, eps, ms, bs)
    secs = time.time() - t0
    return {
        "n": n, "d": d, "eps": [float(e) for e in eps], "min_samples": ms,
        "max_bytes_per_batch": cfg["budget"], "neigh_per_row": cfg["npr"], "index_bits": bits,
        "batch_size": int(bs), "batches": int(-(-n // bs)),
        "points_sha256": hashlib.sha256(pts.tobytes()).hexdigest(),
        "nnz_max_eps": int(nnz), "degree_sum": [int(v) for v in deg.astype(np.int64).sum(axis=1)],
        "configs": summarise(labels, core), "oracle_seconds": round(secs, 1),
        "oracle_threads": oracle.default_threads(),
    }


def main(names: list[str]) -> None:
    data = json.loads(OUT.read_text()) if OUT.exists() else {}
    for name in names:
        print(f"{name}: running the oracle ...", flush=True)
        data[name] = workload(name)
        OUT.write_text(json.dumps(dict(sorted(data.items())), indent=1) + "\n")
        print(f"{name}: done in {data[name]['oracle_seconds']} s", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or ["c1", "c2", "c5", "c3", "c5q", "c4", "c5qb"])
