"""The allocation-free entry point, dbm_neighbor_counts_noalloc, against dbm_neighbor_counts.

Callers that cannot call cudaMalloc (under an allocator that owns all of the device's memory,
or on a path that cannot take cudaMalloc's device-wide synchronisation) use
dbm_neighbor_counts_noalloc, whose scratch is a fixed 32 MiB device array inside the library.  This file is collected last on purpose.  It
calls the new entry point through the C ABI twice in a row on the same inputs and requires
both outputs to equal the allocating entry point's degrees exactly (integer counts, so the
tolerance is zero), then checks that an input too large for the static scratch is refused.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import dbscan_multi as dm

pytestmark = pytest.mark.gpu


def _bind():
    lib = dm.load_library()
    f = lib.dbm_neighbor_counts_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    return f


def _call(f, torch, x, eps):
    e = np.ascontiguousarray(eps, dtype=np.float32)
    deg = torch.full((len(e), x.shape[0]), -7, dtype=torch.int32, device=x.device)
    err = ctypes.create_string_buffer(512)
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(ctypes.c_void_p(x.data_ptr()), x.shape[0], x.shape[1], e.ctypes.data_as(ctypes.c_void_p),
           len(e), ctypes.c_void_p(deg.data_ptr()), ctypes.c_void_p(stream), err, len(err))
    return rc, err.value.decode(), deg


@pytest.mark.parametrize("n,d,eps", [(20_000, 8, [0.6, 0.9, 1.2]), (3_001, 33, [3.0, 4.5]),
                                     (5_000, 2, [0.05, 0.1, 0.2, 0.3])])
def test_noalloc_matches_allocating_entry_point_twice(n, d, eps):
    import torch

    assert torch.cuda.is_available()
    f = _bind()
    rng = np.random.default_rng(n + d)
    c = rng.uniform(-5, 5, size=(max(1, n // 500), d))
    pts = (c[rng.integers(0, len(c), n)] + rng.normal(0, 0.7, (n, d))).astype(np.float32)
    x = torch.from_numpy(pts).cuda()
    with dm.DbscanMulti(0) as h:
        want = h.neighbor_counts(x, eps).cpu().numpy()
    for _ in range(2):
        rc, msg, deg = _call(f, torch, x, eps)
        assert rc == 0, msg
        assert np.array_equal(deg.cpu().numpy(), want)


def test_noalloc_rejects_inputs_beyond_the_static_scratch():
    import torch

    f = _bind()
    x = torch.zeros((1_000_000, 16), dtype=torch.float32, device="cuda")  # needs ~80 MB of scratch
    rc, msg, _ = _call(f, torch, x, [1.0])
    assert rc == -9 and "static scratch" in msg
