"""ctypes front end of the CPU oracle (dbm_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker the CUDA product path is compared against.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module; the product package never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libdbm_oracle.so"
POINTS_TOOL = HERE / "selftest_points"

_lib = None


def build() -> None:
    """Compile the oracle library and the selftest point generator with make."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    lib.dbmo_fit_multi.argtypes = [p, i64, i64, p, i32, p, i32, i64, p, p, p]
    lib.dbmo_fit_multi.restype = i32
    lib.dbmo_fit_multi_stream.argtypes = [p, i64, i64, p, i32, p, i32, i64, p, p, p, i32, p]
    lib.dbmo_fit_multi_stream.restype = i32
    lib.dbmo_codes_degrees.argtypes = [p, i64, i64, p, i32, i64, i64, p, p, i32]
    lib.dbmo_codes_degrees.restype = i32
    lib.dbmo_pair_chain.argtypes = [p, p, i64, i64, p]
    lib.dbmo_pair_chain.restype = None
    lib.dbmo_square_eps.argtypes = [p, i32, p]
    lib.dbmo_square_eps.restype = None
    lib.dbmo_annotate_pays.argtypes = [i64, i64, i32, i64]
    lib.dbmo_annotate_pays.restype = i32
    lib.dbmo_default_threads.argtypes = []
    lib.dbmo_default_threads.restype = i32
    _lib = lib
    return lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def square_eps(eps) -> np.ndarray:
    lib = _load()
    e = np.ascontiguousarray(eps, dtype=np.float32)
    out = np.empty_like(e)
    lib.dbmo_square_eps(_ptr(e), len(e), _ptr(out))
    return out


def fit_multi(points, eps, min_samples, batch_size: int | None = None):
    """Labels (k*l, N) int32, core masks (k*l, N) bool and degrees (k, N) int32.

    ``eps`` and ``min_samples`` must already be ascending and unique (the reference's CLI
    normalises them before calling fit_multi).  ``batch_size`` defaults to N (one batch).
    """
    lib = _load()
    x = np.ascontiguousarray(points, dtype=np.float32)
    n, d = x.shape
    e = np.ascontiguousarray(eps, dtype=np.float32)
    m = np.ascontiguousarray(min_samples, dtype=np.int32)
    k, l = len(e), len(m)
    bs = n if batch_size is None else int(batch_size)
    labels = np.empty((k * l, n), dtype=np.int32)
    core = np.empty((k * l, n), dtype=np.uint8)
    deg = np.empty((k, n), dtype=np.int32)
    rc = lib.dbmo_fit_multi(_ptr(x), n, d, _ptr(e), k, _ptr(m), l, bs, _ptr(labels), _ptr(core), _ptr(deg))
    if rc != 0:
        raise RuntimeError(f"dbmo_fit_multi failed with {rc}")
    return labels, core.astype(bool), deg


def fit_multi_stream(points, eps, min_samples, batch_size: int | None = None, threads: int = 0):
    """The same labels, core masks and degrees as fit_multi, computed batch by batch with only
    one batch's neighbour lists in memory (the reference's own two-pass structure), on
    `threads` host threads (0 = all).  Returns (labels, core, deg, nnz), nnz = the max-eps list
    entries summed over batches (self pairs included)."""
    lib = _load()
    x = np.ascontiguousarray(points, dtype=np.float32)
    n, d = x.shape
    e = np.ascontiguousarray(eps, dtype=np.float32)
    m = np.ascontiguousarray(min_samples, dtype=np.int32)
    k, l = len(e), len(m)
    bs = n if batch_size is None else int(batch_size)
    labels = np.empty((k * l, n), dtype=np.int32)
    core = np.empty((k * l, n), dtype=np.uint8)
    deg = np.empty((k, n), dtype=np.int32)
    nnz = ctypes.c_int64(0)
    rc = lib.dbmo_fit_multi_stream(_ptr(x), n, d, _ptr(e), k, _ptr(m), l, bs, _ptr(labels), _ptr(core), _ptr(deg),
                                   int(threads), ctypes.byref(nnz))
    if rc != 0:
        raise RuntimeError(f"dbmo_fit_multi_stream failed with {rc}")
    return labels, core.astype(bool), deg, int(nnz.value)


def codes_degrees(points, eps, row0: int = 0, rows: int | None = None, want_codes: bool = True,
                  threads: int = 0):
    """Per-pair codes (rows, N) uint8 (255 = none) and cumulative degrees (k, rows)."""
    lib = _load()
    x = np.ascontiguousarray(points, dtype=np.float32)
    n, d = x.shape
    r = n - row0 if rows is None else int(rows)
    eps2 = square_eps(eps)
    k = len(eps2)
    deg = np.empty((k, r), dtype=np.int32)
    codes = np.empty((r, n), dtype=np.uint8) if want_codes else None
    rc = lib.dbmo_codes_degrees(_ptr(x), n, d, _ptr(eps2), k, row0, r, _ptr(deg),
                                _ptr(codes) if codes is not None else None, threads)
    if rc != 0:
        raise RuntimeError(f"dbmo_codes_degrees failed with {rc}")
    return codes, deg


def pair_chain(a, b) -> np.ndarray:
    """The reference's fp32 value acc(a_i, b_i) (sequential fma over the dims) for each row pair
    of two (m, d) arrays."""
    lib = _load()
    x = np.ascontiguousarray(a, dtype=np.float32)
    y = np.ascontiguousarray(b, dtype=np.float32)
    if x.ndim == 1:
        x, y = x[None], y[None]
    out = np.empty(x.shape[0], dtype=np.float32)
    lib.dbmo_pair_chain(_ptr(x), _ptr(y), x.shape[0], x.shape[1], _ptr(out))
    return out


def annotate_pays(nnz: int, pairs: int, k: int, d: int) -> bool:
    return bool(_load().dbmo_annotate_pays(nnz, pairs, k, d))


def default_threads() -> int:
    return int(_load().dbmo_default_threads())


def selftest_points(n_per_cluster: int, d: int, seed: int = 42) -> np.ndarray:
    """The reference selftest's make_blobs points, drawn with the same std:: engine."""
    if not POINTS_TOOL.exists():
        build()
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "p.f32")
        subprocess.run([str(POINTS_TOOL), str(n_per_cluster), str(d), str(seed), out], check=True)
        return np.fromfile(out, dtype=np.float32).reshape(3 * n_per_cluster, d)
