"""C-ABI checks that need no GPU: the library loads, exports every function include/dbm.h
declares, and its host-side rules (batch sizing, route rule, index width) equal the
oracle's restatement of the reference's rules."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

import batching
import dbscan_multi as dm
import oracle

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "dbm.h").read_text()
    return sorted(set(re.findall(r"\b(dbm_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = dm.load_library()
    declared = declared_functions()
    assert set(declared) == set(dm.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(dm.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (dbm_\w+)", out))
    assert set(declared) <= exported


def test_build_info_is_json_with_identity():
    import json

    info = json.loads(dm.build_info())
    assert info["cuda_arch"] == "sm_100a"
    assert info["configured_backend"] in {"cuvs", "codes"}
    assert set(info["compiled_backends"]) == {"cuvs", "codes"}


@pytest.mark.parametrize("n", [1, 7, 1000, 3000, 46340, 46341, 100_000, 1_000_000])
@pytest.mark.parametrize("k,l", [(1, 1), (2, 2), (3, 3), (4, 4), (16, 5)])
@pytest.mark.parametrize("backend", ["cuvs", "codes"])
@pytest.mark.parametrize("npr", [0, 1, 64])
def test_batch_size_matches_reference_rule(n, k, l, backend, npr):
    bits = 64 if n * n >= 2**31 - 1 else 32
    for budget in (1_000_000, 50_000_000, 10**12, 144 * 10**9):
        try:
            want = batching.compute_batch_size(n, k, l, budget, backend == "cuvs", npr, bits)
        except ValueError:
            with pytest.raises(dm.DbmError):
                dm.batch_size(n, k, l, budget, backend, npr)
            continue
        assert dm.batch_size(n, k, l, budget, backend, npr) == want


def test_fixed_buffer_error_code():
    with pytest.raises(dm.DbmError) as ei:
        dm.batch_size(1_000_000, 4, 4, 1000, "cuvs")
    assert ei.value.code == -2


def test_index_overflow_rule():
    # int32 forced at N = 2^31 - 1 leaves (MAX-1)/N = 0 rows
    with pytest.raises(dm.DbmError) as ei:
        dm.batch_size(2**31 - 1, 1, 1, 2**62, "cuvs", 0, "int32")
    assert ei.value.code == -3


def test_max_bytes_inverse():
    for n, k, l, rows, backend in [(3000, 3, 3, 750, "cuvs"), (1000, 2, 2, 98, "codes"), (10**6, 4, 4, 250_000, "cuvs")]:
        b = dm.max_bytes_for_batch_size(n, k, l, rows, backend)
        assert b == batching.max_bytes_for_batch_size(n, k, l, rows, backend == "cuvs", 0,
                                                      64 if n * n >= 2**31 - 1 else 32)
        assert dm.batch_size(n, k, l, b, backend) == rows


@pytest.mark.parametrize("nnz,pairs,k,d", [(4_000_000, 16_000_000, 5, 2), (13_400_000, 64_000**2, 5, 64),
                                           (72_000_000, 16_000 * 64_000, 5, 64), (1_170_000_000, 64_000**2, 5, 64),
                                           (0, 1, 2, 1), (10**12, 10**12, 16, 1000)])
def test_route_rule_matches_oracle(nnz, pairs, k, d):
    assert dm.annotate_pays(nnz, pairs, k, d) == oracle.annotate_pays(nnz, pairs, k, d)


def test_auto_index_bits():
    lib = dm.load_library()
    assert lib.dbm_auto_index_bits(46340) == 32
    assert lib.dbm_auto_index_bits(46341) == 64


def test_list_normalisation_mirrors_cli():
    with pytest.warns(UserWarning):
        e = dm.normalize_eps([0.5, 0.2, 0.5])
    assert e.tolist() == [pytest.approx(0.2), pytest.approx(0.5)]
    with pytest.raises(dm.DbmError):
        dm.normalize_eps([0.0])
    with pytest.raises(dm.DbmError):
        dm.normalize_eps([float("inf")])
    with pytest.raises(dm.DbmError):
        dm.normalize_eps([0.1 * (i + 1) for i in range(17)])
    with pytest.raises(dm.DbmError):
        dm.normalize_min_samples([0, 3])
