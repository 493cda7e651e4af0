"""Runs the reference's own validation gate over this repository's CLI outputs and writes the
verdict to tests/golden/validation_gate.json.

Inputs: tests/golden/cli_labels/<case>.cli_labels.npz, the label files the `dbscan_multi` CLI
wrote on a B200 for the 13 golden cases, one array per mode of the reference's validation matrix
(tools/run_validation_matrix.py:309-320; the GPU test tests/test_cli.py records them when
DBM_RECORD_DIR is set), and each case's points / eps / minPts from tests/golden/<case>.npz.
Gate: `validate_matrix` of the reference (tools/validate_dbscan_matrix.py:175-239): every
configuration of every mode against its float64 DBSCAN oracle (tools/dbscan_validation.py), and
every pair of modes against each other, with the reference's own rules for ambiguous borders.

    python tests/golden/run_validation_gate.py <reference checkout>
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def gate(reference_root: str | Path) -> dict:
    tools = Path(reference_root) / "tools"
    sys.path.insert(0, str(tools))
    try:
        from validate_dbscan_matrix import validate_matrix
    finally:
        sys.path.remove(str(tools))
    out = {}
    for rec in sorted((HERE / "cli_labels").glob("*.cli_labels.npz")):
        case = rec.name.split(".")[0]
        z = np.load(HERE / f"{case}.npz")
        labels = dict(np.load(rec))
        eps = [float(v) for v in z["eps"]]
        ms = [int(v) for v in z["min_samples"]]
        v = validate_matrix(np.asarray(z["points"]), eps, ms, labels, max_n=max(5000, len(z["points"])))
        out[case] = {"modes": sorted(labels), "validacao_aprovada": bool(v["validacao_aprovada"]),
                     "configs": [bool(c["aprovada"]) for c in v["configuracoes"]]}
    return out


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    res = gate(sys.argv[1])
    (HERE / "validation_gate.json").write_text(json.dumps(res, indent=1) + "\n")
    print({k: v["validacao_aprovada"] for k, v in res.items()})
