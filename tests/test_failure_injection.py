"""Failure detection without a GPU fault: the labelling's union-find hooks have a retry bound,
and a test knob (dbm_set_union_retry_limit, like the reference's own test knobs
csr_teto_de_teste / rota_forcada, runner_multi.cuh:145-160, 426-430) lowers it so the bound runs
out at once.  The fit must report DBM_ERR_NOT_CONVERGED through the error word the kernels set,
and the same handle must fit correctly afterwards.  Nothing here can hang: with the bound at 0
every hook returns immediately."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import dbscan_multi as dm
import oracle


def test_union_retry_limit_rejects_a_null_handle_and_negative_limits():
    lib = dm.load_library()
    assert lib.dbm_set_union_retry_limit(None, 0) == -1
    assert lib.dbm_set_union_retry_limit(ctypes.c_void_p(0), 5) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("batched", [False, True])
def test_union_retry_bound_runs_out_and_the_handle_stays_usable(batched):
    import torch

    assert torch.cuda.is_available()
    rng = np.random.default_rng(77)
    c = rng.uniform(-6, 6, size=(5, 3))
    pts = (c[rng.integers(0, 5, 3000)] + rng.normal(0, 0.4, (3000, 3))).astype(np.float32)
    eps, ms = [0.3, 0.5], [4, 9]
    kw = {"max_bytes_per_batch": dm.max_bytes_for_batch_size(3000, 2, 2, 700)} if batched else {}
    x = torch.from_numpy(pts).cuda()
    with dm.DbscanMulti(0) as h:
        with pytest.raises(dm.DbmError):
            h.set_union_retry_limit(-1)
        h.set_union_retry_limit(0)
        with pytest.raises(dm.DbmError) as info:
            h.fit_multi(x, eps, ms, **kw)
        assert info.value.code == -7 and "union-find" in str(info.value)
        h.set_union_retry_limit(1 << 20)
        r = h.fit_multi(x, eps, ms, **kw)
        want, _, _ = oracle.fit_multi(pts, eps, ms, r.stats["batch_size"])
        assert np.array_equal(r.labels.cpu().numpy(), want)
        assert r.stats["batches"] == (5 if batched else 1)
