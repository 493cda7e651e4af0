"""Extracts the reference's golden label bundles into small fixtures for the GPU tests.

The reference ships 13 adversarial cases with the labels its own binary produced in every
mode (cuVS auto/annotated/dense/int64/batched, codes int32/int64/batched, cuML), all of
them raw-equal per case.  The GPU box has no copy of the reference, so this script keeps,
per case: points, eps, min_samples, the labels (one array, after checking that every mode
agrees) and the batch sizes the reference's 1 MB "batched" modes ran with.

It also records the reference selftest's known answers (clusters and noise per
configuration) as read from the shipped selftest log.

Run from the repository root, in a container that has the reference mounted:
    python tests/golden/make_fixtures.py /root/reference
"""

from __future__ import annotations

import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
VALIDATION = "official-campaign-v1/results/pilot-20260817T135424Z/validation"


def main(reference_root: str) -> None:
    src = Path(reference_root) / VALIDATION
    bundles = sorted(src.glob("matrix.*.labels.npz"))
    if len(bundles) != 13:
        raise SystemExit(f"expected 13 golden bundles under {src}, found {len(bundles)}")
    index = []
    for path in bundles:
        z = np.load(path)
        keys = [k for k in z.files if k.startswith("labels_")]
        first = z[keys[0]]
        for key in keys[1:]:
            if not np.array_equal(first, z[key]):
                raise SystemExit(f"{path.name}: mode {key} disagrees with {keys[0]}")
        name = path.name[len("matrix."):-len(".labels.npz")]
        out = HERE / f"{name}.npz"
        np.savez_compressed(
            out,
            points=np.ascontiguousarray(z["points"], dtype=np.float32),
            eps=np.asarray(z["eps"], dtype=np.float64),
            min_samples=np.asarray(z["min_samples"], dtype=np.int64),
            labels=np.asarray(first, dtype=np.int32),
        )
        index.append({"case": name, "file": out.name, "modes_agreeing": sorted(keys)})

    log = (src / "selftest-cuvs.log").read_text(encoding="utf-8")
    answers = []
    for m in re.finditer(r"\[selftest\] eps=([0-9.]+) minPts=(\d+) clusters=(\d+) ruido=(\d+)", log):
        answers.append({"eps": float(m.group(1)), "min_samples": int(m.group(2)),
                        "clusters": int(m.group(3)), "noise": int(m.group(4))})
    batches = re.search(r"lotes: (\d+) x (\d+) pontos", log)
    selftest = {
        "source": f"{VALIDATION}/selftest-cuvs.log",
        "points": "make_blobs(n_per_cluster=1000, d=2, seed=42)",
        "eps": [0.3, 0.5, 0.8],
        "min_samples": [4, 8, 16],
        "configurations": answers,
        "forced_batches": int(batches.group(1)),
        "forced_batch_size": int(batches.group(2)),
    }
    (HERE / "selftest_answers.json").write_text(json.dumps(selftest, indent=1) + "\n")
    (HERE / "index.json").write_text(json.dumps(index, indent=1) + "\n")
    print(f"wrote {len(index)} fixtures and selftest_answers.json to {HERE}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
