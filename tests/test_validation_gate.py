"""The reference's own validation gate over this repository's CLI outputs (no GPU).

tests/golden/cli_labels/ holds the label files the `dbscan_multi` CLI wrote on a B200 for the 13
golden cases in the modes of the reference's validation matrix (tools/run_validation_matrix.py:
309-320); tests/golden/validation_gate.json holds the verdict of the reference's
`validate_matrix` (tools/validate_dbscan_matrix.py:175-239: each mode against the float64 DBSCAN
oracle of tools/dbscan_validation.py, and every pair of modes), written by
tests/golden/run_validation_gate.py.  With DBM_REFERENCE_ROOT pointing at a reference checkout
the gate is run again here, live.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
RECORDS = sorted((GOLDEN / "cli_labels").glob("*.cli_labels.npz"))


def test_every_golden_case_has_recorded_cli_outputs():
    cases = sorted(p.stem for p in GOLDEN.glob("0*.npz"))
    assert [r.name.split(".")[0] for r in RECORDS] == cases


@pytest.mark.parametrize("rec", RECORDS, ids=lambda p: p.name.split(".")[0])
def test_recorded_cli_labels_equal_the_reference_goldens(rec):
    case = rec.name.split(".")[0]
    want = np.load(GOLDEN / f"{case}.npz")["labels"]
    got = dict(np.load(rec))
    assert len(got) >= 2
    for mode, labels in got.items():
        assert np.array_equal(labels, want), mode


def test_recorded_verdict_of_the_reference_gate_approves_every_case():
    verdict = json.loads((GOLDEN / "validation_gate.json").read_text())
    assert sorted(verdict) == [r.name.split(".")[0] for r in RECORDS]
    for case, v in verdict.items():
        assert v["validacao_aprovada"] and all(v["configs"]), case
        assert sorted(v["modes"]) == sorted(np.load(GOLDEN / "cli_labels" / f"{case}.cli_labels.npz").files)


@pytest.mark.skipif(not os.environ.get("DBM_REFERENCE_ROOT"), reason="reference checkout not mounted (DBM_REFERENCE_ROOT)")
def test_reference_gate_live():
    import importlib.util

    spec = importlib.util.spec_from_file_location("run_validation_gate", GOLDEN / "run_validation_gate.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    res = mod.gate(os.environ["DBM_REFERENCE_ROOT"])
    assert res == json.loads((GOLDEN / "validation_gate.json").read_text())
