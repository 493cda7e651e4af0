"""Host side of the B200 multi-parameter DBSCAN: ctypes over libdbm.so (include/dbm.h).

Mirrors the reference's entry point ``ML::Dbscan::Multi::fit_multi``
(src/multi/runner_multi.cuh:1290-1307) and its CLI's argument handling
(src/main.cu:1361-1423):

    fit_multi(x, eps, min_samples, max_bytes_per_batch=0, backend="cuvs", index="auto",
              route="auto", neigh_per_row=0) -> FitResult(labels, core, stats, routes)

* ``x`` is an (N, D) float32 torch tensor on a CUDA device (device path, no copies) or a
  NumPy array (host path: the library copies it in and the labels out).
* ``eps`` / ``min_samples`` are sorted and de-duplicated first, as the reference CLI does
  (``normalize_list``); the configuration order is eps-major, config = e * l + m.
* labels come back as a (k*l, N) int32 array/tensor with -1 for noise; ``core`` holds the
  k*l core masks (uint8).

There is no CPU path: if libdbm.so is missing or no sm_100 device is present, the calls
raise.  PyTorch is used only for device buffers and streams.
"""

from __future__ import annotations

import ctypes
import math
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Sequence

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libdbm.so"

DBM_OK = 0
ERRORS = {
    -1: "DBM_ERR_INVALID",
    -2: "DBM_ERR_FIXED_BUFFERS",
    -3: "DBM_ERR_INDEX_OVERFLOW",
    -4: "DBM_ERR_CSR_NOT_FIT",
    -5: "DBM_ERR_CUDA",
    -6: "DBM_ERR_OOM",
    -7: "DBM_ERR_NOT_CONVERGED",
    -8: "DBM_ERR_NO_DEVICE",
    -9: "DBM_ERR_TOO_LARGE",
    -10: "DBM_ERR_NONFINITE",
}
BACKENDS = {"cuvs": 0, "codes": 1}
ROUTES = {"auto": 0, "annotated": 1, "dense": 2}
INDEX = {"auto": 0, "int32": 32, "int64": 64}
ROUTE_NAMES = {0: "not-applicable", 1: "annotated", 2: "dense"}
MAX_EPS = 16

# every symbol include/dbm.h declares
DISTANCE_MODES = {"auto": 0, "exact": 1, "screened": 2}
GRAPH_MODES = {"auto": 0, "oneshot": 1, "streamed": 2}

EXPORTED = (
    "dbm_create", "dbm_destroy", "dbm_workspace_bytes", "dbm_set_phase_timing", "dbm_set_distance_mode", "dbm_core_sample_indices",
    "dbm_fit_multi", "dbm_fit_multi_host", "dbm_neighbor_counts", "dbm_batch_size", "dbm_max_bytes_for_batch_size",
    "dbm_annotate_pays", "dbm_auto_index_bits", "dbm_build_info_json",
    "dbm_neighbor_counts_noalloc", "dbm_distance_shard", "dbm_fit_multi_from_graph",
    "dbm_set_union_retry_limit", "dbm_set_graph_mode",
    "dbm_prune_units", "dbm_prune_mask_words", "dbm_distance_prune_units", "dbm_distance_shard_pruned",
)


class DbmError(RuntimeError):
    def __init__(self, code: int, message: str):
        self.code = code
        self.name = ERRORS.get(code, f"DBM_ERR_{code}")
        super().__init__(f"{self.name}: {message}")


class Options(ctypes.Structure):
    _fields_ = [
        ("backend", ctypes.c_int),
        ("index_bits", ctypes.c_int),
        ("route", ctypes.c_int),
        ("neigh_per_row", ctypes.c_int64),
        ("max_bytes_per_batch", ctypes.c_uint64),
        ("csr_cap_bytes", ctypes.c_uint64),
    ]


class Stats(ctypes.Structure):
    _fields_ = [
        ("max_bytes_per_batch", ctypes.c_uint64),
        ("batch_size", ctypes.c_uint64),
        ("batches", ctypes.c_int32),
        ("attempts", ctypes.c_int32),
        ("batch_corrections", ctypes.c_int32),
        ("dense_batches", ctypes.c_int32),
        ("annotated_batches", ctypes.c_int32),
        ("index_bits", ctypes.c_int32),
        ("max_nnz", ctypes.c_int64),
        ("total_nnz_max_eps", ctypes.c_int64),
        ("unique_pairs", ctypes.c_int64),
        ("edges", ctypes.c_int64),
        ("distance_passes", ctypes.c_int32),
        ("launches", ctypes.c_int32),
        ("ms_distance", ctypes.c_double),
        ("ms_graph", ctypes.c_double),
        ("ms_label", ctypes.c_double),
        ("ms_relabel", ctypes.c_double),
        ("dist_work_fraction", ctypes.c_double),
        ("tile_pairs_kept", ctypes.c_double),
        ("screened_tile_pairs", ctypes.c_int64),
        ("fallback_tile_pairs", ctypes.c_int64),
        ("screen_candidates", ctypes.c_int64),
        ("ms_screen", ctypes.c_double),
        ("streamed", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_uint64),
        ("nnz_per_eps", ctypes.c_int64 * MAX_EPS),
    ]

    def as_dict(self) -> dict[str, Any]:
        out = {name: getattr(self, name) for name, _ in self._fields_}
        out["nnz_per_eps"] = list(self.nnz_per_eps)
        return out


_lib = None

# cudaStreamLegacy: the legacy default stream as a stream handle.  A torch stream whose handle is 0
# is that stream; 0 itself (NULL) would mean "the handle's own stream" to the C ABI.
CUDA_STREAM_LEGACY = 1


def stream_arg(s: int) -> ctypes.c_void_p:
    """A torch stream handle as the C ABI's `stream` argument, preserving the legacy default
    stream (handle 0) so the library's work is ordered with torch's on that stream."""
    return ctypes.c_void_p(int(s) if s else CUDA_STREAM_LEGACY)


def load_library():
    """Loads libdbm.so; raises if it has not been built (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with cuml-dbscanmulti_b200/build.py")
    lib = ctypes.CDLL(str(LIB_PATH))
    p, i64, u64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_int
    cp, sz = ctypes.c_char_p, ctypes.c_size_t
    lib.dbm_create.argtypes = [i32, p, cp, sz]
    lib.dbm_create.restype = p
    lib.dbm_destroy.argtypes = [p]
    lib.dbm_destroy.restype = None
    lib.dbm_workspace_bytes.argtypes = [p]
    lib.dbm_workspace_bytes.restype = u64
    lib.dbm_set_phase_timing.argtypes = [p, i32]
    lib.dbm_set_phase_timing.restype = None
    lib.dbm_set_distance_mode.argtypes = [p, i32]
    lib.dbm_set_distance_mode.restype = i32
    lib.dbm_set_graph_mode.argtypes = [p, i32]
    lib.dbm_set_graph_mode.restype = i32
    lib.dbm_set_union_retry_limit.argtypes = [p, i32]
    lib.dbm_set_union_retry_limit.restype = i32
    lib.dbm_core_sample_indices.argtypes = [p, p, i64, i32, p, p, cp, sz]
    lib.dbm_core_sample_indices.restype = i32
    fit_args = [p, p, i64, i64, p, i32, p, i32, p, p, ctypes.POINTER(Options), ctypes.POINTER(Stats),
                p, i32]
    lib.dbm_fit_multi.argtypes = fit_args + [p, cp, sz]
    lib.dbm_fit_multi.restype = i32
    lib.dbm_fit_multi_host.argtypes = fit_args + [cp, sz]
    lib.dbm_fit_multi_host.restype = i32
    lib.dbm_distance_shard.argtypes = [p, p, i64, i64, p, i32, i32, i32, p, p, u64, ctypes.POINTER(u64),
                                       ctypes.POINTER(Stats), p, cp, sz]
    lib.dbm_distance_shard.restype = i32
    lib.dbm_prune_units.argtypes = [i64]
    lib.dbm_prune_units.restype = i64
    lib.dbm_prune_mask_words.argtypes = []
    lib.dbm_prune_mask_words.restype = i32
    lib.dbm_distance_prune_units.argtypes = [p, p, i64, i64, p, i32, i64, i64, p, p, p, cp, sz]
    lib.dbm_distance_prune_units.restype = i32
    lib.dbm_distance_shard_pruned.argtypes = [p, p, i64, i64, p, i32, i32, i32, p, p, p, p, u64, ctypes.POINTER(u64),
                                              ctypes.POINTER(Stats), p, cp, sz]
    lib.dbm_distance_shard_pruned.restype = i32
    lib.dbm_fit_multi_from_graph.argtypes = [p, i64, i64, p, i32, p, i32, p, p, u64, i32, i32, p, p,
                                             ctypes.POINTER(Options), ctypes.POINTER(Stats), p, i32, p, cp, sz]
    lib.dbm_fit_multi_from_graph.restype = i32
    lib.dbm_neighbor_counts.argtypes = [p, p, i64, i64, p, i32, p, p, cp, sz]
    lib.dbm_neighbor_counts.restype = i32
    lib.dbm_batch_size.argtypes = [i64, i32, i32, u64, i32, i64, i32, ctypes.POINTER(u64), cp, sz]
    lib.dbm_batch_size.restype = i32
    lib.dbm_max_bytes_for_batch_size.argtypes = [i64, i32, i32, u64, i32, i64, i32]
    lib.dbm_max_bytes_for_batch_size.restype = u64
    lib.dbm_annotate_pays.argtypes = [i64, i64, i32, i64]
    lib.dbm_annotate_pays.restype = i32
    lib.dbm_auto_index_bits.argtypes = [i64]
    lib.dbm_auto_index_bits.restype = i32
    lib.dbm_build_info_json.argtypes = []
    lib.dbm_build_info_json.restype = ctypes.c_char_p
    _lib = lib
    return lib


def build_info() -> str:
    return load_library().dbm_build_info_json().decode()


# ---- list normalisation (src/main.cu:428-439, 1397-1417) ---------------------------------------
def normalize_eps(eps: Sequence[float]) -> np.ndarray:
    vals = np.asarray([np.float32(v) for v in eps], dtype=np.float32)
    out = np.unique(vals)
    if out.size != vals.size or not np.array_equal(out, vals):
        warnings.warn("eps was sorted/de-duplicated; configuration order follows the result's eps")
    if out.size == 0 or out.size > MAX_EPS:
        raise DbmError(-1, f"between 1 and {MAX_EPS} eps values are required")
    safe = np.float32(math.sqrt(np.finfo(np.float32).max))
    if not np.all(np.isfinite(out)) or np.any(out <= 0) or np.any(out > safe):
        raise DbmError(-1, "eps values must be finite, positive and not overflow eps^2")
    return out


def normalize_min_samples(min_samples: Sequence[int]) -> np.ndarray:
    vals = np.asarray([int(v) for v in min_samples], dtype=np.int64)
    out = np.unique(vals)
    if out.size != vals.size or not np.array_equal(out, vals):
        warnings.warn("min_samples was sorted/de-duplicated; configuration order follows the result's min_samples")
    if out.size == 0 or np.any(out <= 0) or np.any(out > np.iinfo(np.int32).max):
        raise DbmError(-1, "min-samples values must be positive int32 values")
    return out.astype(np.int32)


def batch_size(n: int, k: int, l: int, max_bytes: int, backend: str = "cuvs", neigh_per_row: int = 0,
               index: str = "auto") -> int:
    """The reference's compute_batch_size_multi (runner_multi.cuh:458-499)."""
    lib = load_library()
    out = ctypes.c_uint64(0)
    err = ctypes.create_string_buffer(512)
    rc = lib.dbm_batch_size(n, k, l, max_bytes, BACKENDS[backend], neigh_per_row, INDEX[index],
                            ctypes.byref(out), err, len(err))
    if rc != DBM_OK:
        raise DbmError(rc, err.value.decode())
    return int(out.value)


def max_bytes_for_batch_size(n: int, k: int, l: int, rows: int, backend: str = "cuvs",
                             neigh_per_row: int = 0, index: str = "auto") -> int:
    return int(load_library().dbm_max_bytes_for_batch_size(n, k, l, rows, BACKENDS[backend],
                                                           neigh_per_row, INDEX[index]))


def annotate_pays(nnz: int, pairs: int, k: int, d: int) -> bool:
    return bool(load_library().dbm_annotate_pays(nnz, pairs, k, d))


@dataclass
class FitResult:
    labels: Any                     # (k*l, N) int32 (torch tensor on device, or numpy)
    core: Any                       # (k*l, N) uint8 or None
    eps: np.ndarray
    min_samples: np.ndarray
    stats: dict[str, Any] = field(default_factory=dict)
    batch_routes: list[str] = field(default_factory=list)
    index: str = "int32"
    backend: str = "cuvs"

    @property
    def route_observed(self) -> str:
        if self.backend != "cuvs" or len(self.eps) <= 1:
            return "not-applicable"
        a = self.batch_routes.count("annotated")
        d = self.batch_routes.count("dense")
        return "mixed" if a and d else "annotated" if a else "dense" if d else "not-applicable"


class DbscanMulti:
    """A device-bound handle: stream + persistent workspace reused across fits
    (the reference's workspace_externo + BuffersCsr, runner_multi.cuh:516-526)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        self._lib = load_library()
        err = ctypes.create_string_buffer(512)
        self._h = self._lib.dbm_create(int(device), ctypes.c_void_p(stream) if stream else None, err, len(err))
        if not self._h:
            raise DbmError(-8, err.value.decode())
        self.device = int(device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.dbm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def workspace_bytes(self) -> int:
        return int(self._lib.dbm_workspace_bytes(self._h))

    def set_phase_timing(self, enabled: bool) -> None:
        self._lib.dbm_set_phase_timing(self._h, 1 if enabled else 0)

    def set_distance_mode(self, mode: str) -> None:
        """'auto' (tensor-core screen where it applies), 'exact' (exact tile kernel only) or
        'screened' (require the screen).  Labels are identical in every mode."""
        rc = self._lib.dbm_set_distance_mode(self._h, DISTANCE_MODES[mode])
        if rc != DBM_OK:
            raise DbmError(rc, f"bad distance mode {mode!r}")

    def set_graph_mode(self, mode: str) -> None:
        """'auto' (the whole graph at once when it fits the budget and the free memory, else one
        row batch at a time), 'oneshot' or 'streamed'.  Labels are identical in every mode."""
        rc = self._lib.dbm_set_graph_mode(self._h, GRAPH_MODES[mode])
        if rc != DBM_OK:
            raise DbmError(rc, f"bad graph mode {mode!r}")

    def set_union_retry_limit(self, limit: int) -> None:
        """Test knob: the retry bound of every union-find hook (default 2**20; 0 makes the
        labelling give up with DBM_ERR_NOT_CONVERGED).  The handle stays usable."""
        rc = self._lib.dbm_set_union_retry_limit(self._h, int(limit))
        if rc != DBM_OK:
            raise DbmError(rc, f"bad union retry limit {limit!r}")

    def _options(self, backend, index, route, neigh_per_row, max_bytes_per_batch, csr_cap_bytes):
        if backend not in BACKENDS:
            raise DbmError(-1, f"--backend must be 'cuvs' or 'codes', got {backend!r}")
        if index not in INDEX:
            raise DbmError(-1, f"--index must be 'auto', 'int32' or 'int64', got {index!r}")
        if route not in ROUTES:
            raise DbmError(-1, f"--route must be 'auto', 'annotated' or 'dense', got {route!r}")
        if route != "auto" and backend != "cuvs":
            raise DbmError(-1, "--route only applies to the cuvs backend")
        if neigh_per_row < 0:
            raise DbmError(-1, "--neigh-per-row must be >= 0")
        return Options(BACKENDS[backend], INDEX[index], ROUTES[route], int(neigh_per_row),
                       int(max_bytes_per_batch), int(csr_cap_bytes))

    def neighbor_counts(self, x, eps, stream: int | None = None):
        """(k, N) int32 tensor of per-eps neighbourhood sizes (self included) for a CUDA tensor."""
        import torch

        e = normalize_eps(eps)
        if not x.is_cuda or x.dtype != torch.float32 or x.dim() != 2:
            raise DbmError(-1, "x must be a 2-D float32 CUDA tensor")
        x = x.contiguous()
        n, d = int(x.shape[0]), int(x.shape[1])
        deg = torch.empty((len(e), n), dtype=torch.int32, device=x.device)
        s = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        err = ctypes.create_string_buffer(1024)
        rc = self._lib.dbm_neighbor_counts(self._h, ctypes.c_void_p(x.data_ptr()), n, d,
                                           e.ctypes.data_as(ctypes.c_void_p), len(e),
                                           ctypes.c_void_p(deg.data_ptr()), stream_arg(s), err, len(err))
        if rc != DBM_OK:
            raise DbmError(rc, err.value.decode())
        return deg

    def core_sample_indices(self, core, stream: int | None = None):
        """sklearn's core_sample_indices_ for every labelling of a fit: row c holds the indices of
        the core points of configuration c, ascending, then -1 (cuML's convention).  `core` is the
        (configs, N) uint8 core mask of fit_multi(..., return_core=True): a CUDA tensor (result on
        the device) or a numpy array (staged through the device)."""
        import torch

        on_host = not type(core).__module__.startswith("torch")
        c = torch.from_numpy(np.ascontiguousarray(core, dtype=np.uint8)).to(f"cuda:{self.device}") if on_host \
            else core.contiguous()
        if c.dim() != 2 or c.dtype != torch.uint8:
            raise DbmError(-1, "core must be a (configs, N) uint8 mask")
        out = torch.empty(c.shape, dtype=torch.int32, device=c.device)
        s = stream if stream is not None else torch.cuda.current_stream(c.device).cuda_stream
        err = ctypes.create_string_buffer(1024)
        rc = self._lib.dbm_core_sample_indices(self._h, ctypes.c_void_p(c.data_ptr()), int(c.shape[1]),
                                               int(c.shape[0]), ctypes.c_void_p(out.data_ptr()), stream_arg(s),
                                               err, len(err))
        if rc != DBM_OK:
            raise DbmError(rc, err.value.decode())
        return out.cpu().numpy() if on_host else out

    def _routes_buffer(self, size: int):
        """A per-handle route buffer of at least `size` bytes (the library writes only the
        batches' entries, so it is reused without clearing)."""
        buf = getattr(self, "_routes", None)
        if buf is None or len(buf) < size:
            buf = self._routes = (ctypes.c_uint8 * size)()
        return buf

    def fit_multi(self, x, eps, min_samples, *, max_bytes_per_batch: int = 0, backend: str = "cuvs",
                  index: str = "auto", route: str = "auto", neigh_per_row: int = 0,
                  csr_cap_bytes: int = 0, return_core: bool = False, labels_out=None,
                  stream: int | None = None) -> FitResult:
        e = normalize_eps(eps)
        m = normalize_min_samples(min_samples)
        k, l = len(e), len(m)
        opt = self._options(backend, index, route, neigh_per_row, max_bytes_per_batch, csr_cap_bytes)
        st = Stats()
        err = ctypes.create_string_buffer(1024)
        is_torch = type(x).__module__.startswith("torch")
        if is_torch:
            import torch

            if not x.is_cuda or x.dtype != torch.float32 or x.dim() != 2:
                raise DbmError(-1, "x must be a 2-D float32 CUDA tensor")
            x = x.contiguous()
            n, d = int(x.shape[0]), int(x.shape[1])
            maxb = n + 1
            routes = self._routes_buffer(maxb)
            labels = labels_out if labels_out is not None else torch.empty((k * l, n), dtype=torch.int32, device=x.device)
            core = torch.empty((k * l, n), dtype=torch.uint8, device=x.device) if return_core else None
            s = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
            rc = self._lib.dbm_fit_multi(
                self._h, ctypes.c_void_p(x.data_ptr()), n, d, e.ctypes.data_as(ctypes.c_void_p), k,
                m.ctypes.data_as(ctypes.c_void_p), l, ctypes.c_void_p(labels.data_ptr()),
                ctypes.c_void_p(core.data_ptr()) if core is not None else None, ctypes.byref(opt),
                ctypes.byref(st), routes, maxb, stream_arg(s), err, len(err))
        else:
            xh = np.ascontiguousarray(x, dtype=np.float32)
            if xh.ndim != 2:
                raise DbmError(-1, "x must be two-dimensional")
            # NaN/Inf are detected on the device (DBM_ERR_NONFINITE)
            n, d = xh.shape
            maxb = n + 1
            routes = self._routes_buffer(maxb)
            if labels_out is not None:
                labels = labels_out
                if (labels.dtype != np.int32 or labels.shape != (k * l, n)
                        or not labels.flags["C_CONTIGUOUS"]):
                    raise DbmError(-1, "labels_out must be a C-contiguous (k*l, N) int32 array")
            else:
                labels = np.empty((k * l, n), dtype=np.int32)
            core = np.empty((k * l, n), dtype=np.uint8) if return_core else None
            rc = self._lib.dbm_fit_multi_host(
                self._h, xh.ctypes.data_as(ctypes.c_void_p), n, d, e.ctypes.data_as(ctypes.c_void_p), k,
                m.ctypes.data_as(ctypes.c_void_p), l, labels.ctypes.data_as(ctypes.c_void_p),
                core.ctypes.data_as(ctypes.c_void_p) if core is not None else None, ctypes.byref(opt),
                ctypes.byref(st), routes, maxb, err, len(err))
        if rc != DBM_OK:
            raise DbmError(rc, err.value.decode())
        nb = int(st.batches)
        return FitResult(labels=labels, core=core, eps=e, min_samples=m, stats=st.as_dict(),
                         batch_routes=[ROUTE_NAMES[int(routes[i])] for i in range(nb)],
                         index="int64" if st.index_bits == 64 else "int32", backend=backend)


_default: dict[int, DbscanMulti] = {}


def fit_multi(x, eps, min_samples, **kw) -> FitResult:
    """Module-level convenience: one cached handle per device."""
    dev = 0
    if type(x).__module__.startswith("torch") and x.is_cuda:
        dev = x.device.index or 0
    h = _default.get(dev)
    if h is None:
        h = _default[dev] = DbscanMulti(dev)
    return h.fit_multi(x, eps, min_samples, **kw)
