"""The dbscan_multi CLI: the reference CLI's flags, files and last-line JSON contract
(src/main.cu:233-269, 1361-1643), as its Python tools invoke it
(tools/run_validation_matrix.py:51-137, tools/bench_vs_cuml.py:414-490)."""

from __future__ import annotations

import json
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "cuml-dbscanmulti_b200" / "bin" / "dbscan_multi"
GOLDEN = ROOT / "tests" / "golden"
# The reference checkout, when mounted (its tools/ hold the JSON contract validator); the
# checks that need it skip when DBM_REFERENCE_ROOT is unset.
REFERENCE_ROOT = os.environ.get("DBM_REFERENCE_ROOT", "")
REFERENCE_TOOLS = Path(REFERENCE_ROOT) / "tools" if REFERENCE_ROOT else None
# Optional directory where the GPU tests also leave their recorded CLI outputs (JSON lines and
# label files) for tests/golden/ fixtures; unset = tmp_path only.
RECORD_DIR = os.environ.get("DBM_RECORD_DIR", "")


def run(*args, check=False):
    return subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True, check=check)


def last_json(stdout):
    for line in reversed(stdout.splitlines()):
        if line.strip().startswith("{"):
            return json.loads(line)
    raise AssertionError("no JSON line")


# ---- no GPU needed: argument handling exits before any device work -------------------------
def test_cli_built():
    assert CLI.exists(), "build with cuml-dbscanmulti_b200/build.py"


def test_build_info_identity():
    info = last_json(run("--build-info", check=True).stdout)["build"]
    assert re.fullmatch(r"[0-9a-fA-F]{7,64}", info["git_sha"])
    assert info["build_id"] not in ("", "unknown")
    assert set(info["compiled_backends"]) == {"cuvs", "codes"} and info["configured_backend"] == "cuvs"


@pytest.mark.parametrize("args", [
    ["--n", "3"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "0.1", "--min-samples", "2", "--route", "dense",
     "--backend", "codes"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "0.1,,0.2", "--min-samples", "2"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "0.1", "--eps-min", "0.1", "--min-samples", "2"],
    ["--bogus"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "0", "--min-samples", "2"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "0.1", "--min-samples", "0"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "nan", "--min-samples", "2"],
    ["--selftest", "--route", "dense"],
    ["--input", "x", "--n", "3", "--d", "1", "--eps", "0.1", "--min-samples", "2", "--repeat", "0"],
])
def test_usage_errors_exit_2(args):
    assert run(*args).returncode == 2


def test_bad_file_size_exits_1(tmp_path):
    p = tmp_path / "x.f32"
    np.zeros(5, np.float32).tofile(p)
    assert run("--input", p, "--n", 3, "--d", 2, "--eps", 0.1, "--min-samples", 2).returncode == 1


def validate_contract(meta, backend, n, d, eps, min_samples, index, route):
    """Restates the checks of tools/bench_vs_cuml.py:validar_contrato_runtime."""
    assert meta["backend"] == backend
    assert meta["index"] == index if index != "auto" else meta["index"] in ("int32", "int64")
    assert meta["configuration_count"] == len(eps) * len(min_samples)
    assert meta["eps_count"] == len(eps) and meta["min_samples_count"] == len(min_samples)
    want = np.asarray([np.float32(float(f"{v:.10g}")) for v in eps], np.float64)
    assert np.allclose(np.asarray(meta["eps"], np.float64), want, rtol=5e-6, atol=1e-12)
    assert meta["min_samples"] == [int(v) for v in min_samples]
    assert meta["config_order"] == "eps_major" and meta["n"] == n and meta["d"] == d
    assert meta["requested_route"] == route
    ex = meta["execution"]
    assert isinstance(ex["batches"], int) and ex["batches"] > 0
    assert len(ex["batch_routes"]) == ex["batches"]
    a, dn = ex["batch_routes"].count("annotated"), ex["batch_routes"].count("dense")
    assert ex["annotated_batches"] == a and ex["dense_batches"] == dn
    if backend == "cuvs" and len(eps) > 1:
        assert "not-applicable" not in ex["batch_routes"]
        if route in ("annotated", "dense"):
            assert set(ex["batch_routes"]) == {route}
    else:
        assert set(ex["batch_routes"]) == {"not-applicable"}
    observed = "mixed" if a and dn else "annotated" if a else "dense" if dn else "not-applicable"
    assert ex["route_observed"] == observed
    b = meta["build"]
    assert re.fullmatch(r"[0-9a-fA-F]{7,64}", b["git_sha"]) and b["build_id"] not in ("", "unknown")
    assert backend in b["compiled_backends"]


def validate_with_reference_tool(meta, **kw):
    """When the reference's tools are mounted, also run its own validator on the JSON."""
    if REFERENCE_TOOLS is None or not (REFERENCE_TOOLS / "bench_vs_cuml.py").exists():
        return
    sys.path.insert(0, str(REFERENCE_TOOLS))
    try:
        import bench_vs_cuml  # noqa: E402

        bench_vs_cuml.validar_contrato_runtime(meta, **kw)
    finally:
        sys.path.remove(str(REFERENCE_TOOLS))


def test_recorded_cli_json_passes_the_reference_validator():
    """tests/golden/cli_run.json was produced by this CLI on a B200 (see tests/golden/README)."""
    path = GOLDEN / "cli_run.json"
    if not path.exists():
        pytest.skip("no recorded CLI run yet")
    rec = json.loads(path.read_text())
    for entry in rec["runs"]:
        args = entry["request"]
        validate_contract(entry["json"], **args)
        validate_with_reference_tool(entry["json"], backend=args["backend"], n=args["n"], d=args["d"],
                                     eps=args["eps"], min_samples=args["min_samples"], index=args["index"],
                                     route=args["route"])


MODES = [
    dict(backend="cuvs", index="int32", route="auto"),
    dict(backend="cuvs", index="int32", route="annotated"),
    dict(backend="cuvs", index="int32", route="dense"),
    dict(backend="cuvs", index="int64", route="auto"),
    dict(backend="codes", index="int32", route="auto"),
    dict(backend="codes", index="int64", route="auto"),
    dict(backend="cuvs", index="int32", route="auto", max_mbytes=1),
    dict(backend="codes", index="int32", route="auto", max_mbytes=1),
]


# every mode on the cases that stress routes, batching, boundaries and the fallback dims;
# two modes (cuVS auto, codes batched) on the rest -- each CLI process pays CUDA start-up
FULL_MODE_CASES = {"002_ambiguous_border_2d", "003_epsilon_nextafter_1d", "008_high_dimension_8193",
                   "009_forced_batches_2d", "010_random_seed_000"}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("0*.npz")))
def test_cli_golden_bundles_every_mode(tmp_path, name):
    z = np.load(GOLDEN / f"{name}.npz")
    pts = np.ascontiguousarray(z["points"], np.float32)
    eps = sorted({float(v) for v in z["eps"]})
    ms = sorted({int(v) for v in z["min_samples"]})
    pts_path = tmp_path / "p.f32"
    pts.tofile(pts_path)
    runs = []
    recorded = {}
    modes = MODES if name in FULL_MODE_CASES else [MODES[0], MODES[7]]
    for mode in modes:
        out = tmp_path / "l.i32"
        cmd = ["--input", pts_path, "--output", out, "--n", pts.shape[0], "--d", pts.shape[1],
               "--eps", ",".join(format(v, ".10g") for v in eps),
               "--min-samples", ",".join(str(v) for v in ms),
               "--backend", mode["backend"], "--index", mode["index"], "--route", mode["route"],
               "--warmup", 0, "--repeat", 1, "--json"]
        if mode.get("max_mbytes"):
            cmd += ["--max-mbytes-per-batch", mode["max_mbytes"]]
        if mode["route"] != "auto" and mode["backend"] != "cuvs":
            continue
        p = run(*cmd)
        assert p.returncode == 0, p.stderr
        meta = last_json(p.stdout)
        validate_contract(meta, mode["backend"], pts.shape[0], pts.shape[1], eps, ms, mode["index"], mode["route"])
        labels = np.fromfile(out, np.int32).reshape(len(eps) * len(ms), pts.shape[0])
        assert np.array_equal(labels, z["labels"]), mode
        recorded[mode_name(mode)] = labels
        runs.append({"request": dict(backend=mode["backend"], n=int(pts.shape[0]), d=int(pts.shape[1]),
                                     eps=eps, min_samples=ms, index=mode["index"], route=mode["route"]),
                     "json": meta})
    # the label files each mode wrote, kept for the reference's own validation gate
    # (tests/test_validation_gate.py) and, for one case, the JSON lines for its contract validator
    np.savez_compressed(tmp_path / f"{name}.cli_labels.npz", **recorded)
    if name == "010_random_seed_000":
        (tmp_path / "cli_run.json").write_text(json.dumps({"runs": runs}, indent=1))
    if RECORD_DIR:
        dst = Path(RECORD_DIR)
        dst.mkdir(parents=True, exist_ok=True)
        for f in tmp_path.glob("*.json*"):
            (dst / f.name).write_bytes(f.read_bytes())
        (dst / f"{name}.cli_labels.npz").write_bytes((tmp_path / f"{name}.cli_labels.npz").read_bytes())


def mode_name(mode):
    """Name of a CLI mode, as the reference's validation matrix spells its sources."""
    base = f"{mode['backend']}_{mode['route']}_{mode['index']}"
    return base + ("_batched" if mode.get("max_mbytes") else "")


@pytest.mark.gpu
def test_cli_selftest_passes():
    for backend in ("cuvs", "codes"):
        p = run("--selftest", "--backend", backend, "--json")
        assert p.returncode == 0, p.stderr
        meta = last_json(p.stdout)
        assert meta["selftest"] is True
        assert [(c["n_clusters"], c["n_noise"]) for c in meta["configurations"]] == \
            [(3, 22), (3, 35), (3, 70), (3, 2), (3, 2), (3, 4), (3, 0), (3, 0), (3, 0)]
        assert meta["batches"] == 4 and meta["batch_size"] == 750 if backend == "cuvs" else True


@pytest.mark.gpu
def test_cli_solo_and_perfil(tmp_path):
    rng = np.random.default_rng(3)
    pts = np.vstack([rng.normal(c, 0.3, (400, 3)) for c in (0, 3, 6)]).astype(np.float32)
    p_path = tmp_path / "p.f32"
    pts.tofile(p_path)
    p = run("--input", p_path, "--n", len(pts), "--d", 3, "--eps", "0.3,0.5", "--min-samples", "4,8",
            "--warmup", 1, "--repeat", 3, "--solo", "--perfil", "--json")
    assert p.returncode == 0, p.stderr
    meta = last_json(p.stdout)
    assert len(meta["fit_ms_all"]) == 3 and len(meta["solo_ms"]) == 4 and len(meta["solo_ms_all"]) == 4
    assert "[perfil]" in p.stderr
