"""Sharded fit on 2 GPUs (NCCL, one process per GPU) equals the single-GPU fit and the oracle.
Skipped when fewer than two GPUs are visible."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _points(n=20_000, d=8, seed=11):
    rng = np.random.default_rng(seed)
    c = rng.uniform(-6, 6, size=(25, d))
    m = n - n // 20
    pts = c[rng.integers(0, 25, m)] + rng.normal(0, 0.8, (m, d))
    return np.vstack([pts, rng.uniform(-6, 6, (n - m, d))]).astype(np.float32)


EPS = [0.7, 1.0, 1.3]
MS = [4, 9]
ROWS = 3000


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    import dbscan_multi as dm
    from dbscan_multi import parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        pts = _points()
        x = torch.from_numpy(pts).cuda(rank)
        budget = dm.max_bytes_for_batch_size(len(pts), len(EPS), len(MS), ROWS, "cuvs")
        with dm.DbscanMulti(rank) as h:
            stages = parallel.DeviceStages(h)
            res = parallel.sharded_fit_multi(stages, x, EPS, MS, max_bytes_per_batch=budget)
            np.save(os.path.join(out_dir, f"labels_{rank}.npy"), res.labels.cpu().numpy())
            # host points: each rank copies its row slice, an all-gather assembles the rest; the
            # limits agreed once and reused
            limits = parallel.agree_limits(stages, budget, 0, device=torch.device("cuda", rank))
            for _ in range(2):
                res = parallel.sharded_fit_multi(stages, torch.from_numpy(pts).pin_memory(), EPS, MS, limits=limits,
                                                 device=torch.device("cuda", rank), max_bytes_per_batch=budget)
            np.save(os.path.join(out_dir, f"labels_host_{rank}.npy"), res.labels.cpu().numpy())
            torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_fit_matches_single_gpu_and_oracle(tmp_path):
    import torch
    import torch.multiprocessing as mp

    import dbscan_multi as dm
    import oracle

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    pts = _points()
    budget = dm.max_bytes_for_batch_size(len(pts), len(EPS), len(MS), ROWS, "cuvs")
    with dm.DbscanMulti(0) as h:
        single = h.fit_multi(torch.from_numpy(pts).cuda(0), EPS, MS, max_bytes_per_batch=budget).labels.cpu().numpy()
    want, _, _ = oracle.fit_multi(pts, EPS, MS, ROWS)
    assert np.array_equal(single, want)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"labels_{r}.npy"), want)
        assert np.array_equal(np.load(tmp_path / f"labels_host_{r}.npy"), want)
