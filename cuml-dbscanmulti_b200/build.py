"""Builds libdbm.so (sm_100a) and the dbscan_multi CLI in-tree with nvcc.

Outputs (git-ignored, shipped with the source tree):
    dbscan_multi/libdbm.so   the C-ABI library (include/dbm.h)
    bin/dbscan_multi         the command-line front end (same flags and JSON as the
                             reference's CLI)

usage: python cuml-dbscanmulti_b200/build.py [--force]
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "dbscan_multi" / "libdbm.so"
CLI = PKG / "bin" / "dbscan_multi"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def _source_hash() -> str:
    """SHA-256 over the sources (used when no git revision is available)."""
    import hashlib

    h = hashlib.sha256()
    for f in sorted(CSRC.rglob("*")) + [ROOT / "include" / "dbm.h"]:
        if f.is_file() and f.suffix in {".cu", ".cuh", ".cpp", ".h"}:
            h.update(f.relative_to(ROOT).as_posix().encode())
            h.update(f.read_bytes())
    return h.hexdigest()


def _git_sha() -> str:
    try:
        out = subprocess.run(["git", "-C", str(ROOT), "rev-parse", "HEAD"], capture_output=True,
                             text=True, check=True).stdout.strip()
        if out:
            return out
    except Exception:
        pass
    return _source_hash()


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    deps = _sources() + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "dbm.h"]
    if not force and not _stale(LIB, deps):
        return LIB
    sha = _git_sha()
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON, "-shared", "-o", str(LIB),
           f"-DDBM_GIT_SHA=\"{sha}\"", f"-DDBM_BUILD_ID=\"sm_100a-{sha[:12]}\"",
           *[str(s) for s in _sources()]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    LIB.parent.mkdir(parents=True, exist_ok=True)
    subprocess.run(cmd, check=True)
    return LIB


def build_cli(force: bool = False) -> Path:
    src = CSRC / "cli" / "dbscan_multi.cpp"
    if not src.exists():
        return CLI
    deps = [src, ROOT / "include" / "dbm.h", LIB]
    if not force and not _stale(CLI, deps):
        return CLI
    CLI.parent.mkdir(parents=True, exist_ok=True)
    cmd = [_nvcc(), *ARCH_FLAGS, "-O2", "-std=c++17", "-o", str(CLI), str(src), f"-I{ROOT / 'include'}",
           f"-L{LIB.parent}", "-ldbm", "-Xlinker", "-rpath,$ORIGIN/../dbscan_multi"]
    subprocess.run(cmd, check=True)
    return CLI


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_cli(force=force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
