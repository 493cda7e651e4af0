#!/usr/bin/env python
"""Benchmark of the multi-parameter DBSCAN grid fit (fit_multi) on B200.

A "step" is one k x l grid fit over the workload's points: neighbourhood pass, degrees,
core masks, CSR, batched connected components and relabel, labels left on the device.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4] [--impl reference]

Default workload (c4): N=1,000,000, D=33 (32 informative + 1 zero column), 100 Gaussian
blobs (centres U[-20,20]^32, std U[0.8,1.5]) + 5% uniform noise, 4 x 4 grid
eps {3.0,3.5,4.0,4.5} x minPts {5,10,20,40}, a 128 GB budget with neigh_per_row=64
(8 batches of 127,8xx rows).  Seeded synthetic data with the shapes of the published
configuration.

Metric: the k x l grid wall time (`grid_wall_s`, seconds per grid), and as `value` the
effective pair-distances per second = N^2 ordered pairs per grid / grid wall time (the
reference's unit; pairs ruled out by the exact tile bound or the tensor-core screen are resolved
without an fp32 distance evaluation, so this is a rate of pairs resolved, not of distances
computed).  `value` times device-resident input with CUDA events; `e2e` times the host-buffer
C-ABI entry point with the point copy in and the label copy out inside the timed region.
Before timing, the labels are checked against the oracle's digests of the workload and, on
several GPUs, against a one-GPU fit (`labels_match_oracle`, `labels_match_1gpu`; a mismatch
fails the run).

Multi-GPU (torchrun, one process per GPU): the same grid, sharded -- each rank evaluates an
equal share of the distance tile pairs, histograms are all-reduced and neighbour pairs
all-gathered over NCCL, each rank labels a range of the k*l configurations and the labels are
all-gathered (dbscan_multi.parallel).  value = N^2 pairs per grid / max-over-ranks grid time
(fixed total work: strong scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "cuml-dbscanmulti_b200", ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

CONFIGS = {
    "c1": dict(n=10_000, d=2, centers=8, box=10.0, std=(0.5, 0.5), noise=0.05, zero_cols=0,
               eps=[0.2, 0.3, 0.5], min_samples=[5, 10, 20], budget=128 * 10**9, npr=0,
               desc="Gaussian blobs N=10,000 D=2, 8 centres U[-10,10]^2, std 0.5, 5% noise; 3x3 grid"),
    "c2": dict(n=100_000, d=8, centers=20, box=10.0, std=(0.5, 1.0), noise=0.05, zero_cols=0,
               eps=[0.4, 0.6, 0.8, 1.0, 1.2], min_samples=[10], budget=128 * 10**9, npr=0,
               desc="Multi-EPS N=100,000 D=8, 20 centres U[-10,10]^8, std U[0.5,1.0], 5% noise; k=5, l=1"),
    "c3": dict(n=500_000, d=32, centers=50, box=20.0, std=(1.0, 1.0), noise=0.10, zero_cols=0,
               eps=[4.0], min_samples=[5, 10, 20, 40, 80], budget=128 * 10**9, npr=0,
               desc="Multi-minPts N=500,000 D=32, 50 centres U[-20,20]^32, std 1.0, 10% noise; k=1, l=5"),
    "c4": dict(n=1_000_000, d=33, centers=100, box=20.0, std=(0.8, 1.5), noise=0.05, zero_cols=1,
               eps=[3.0, 3.5, 4.0, 4.5], min_samples=[5, 10, 20, 40], budget=128 * 10**9, npr=64,
               desc="Multi-Both N=1,000,000 D=33 (32 informative + 1 zero column), 100 centres "
                    "U[-20,20]^32, std U[0.8,1.5], 5% noise; 4x4 grid; 128 GB budget, "
                    "neigh_per_row 64 -> 8 batches"),
    "c5": dict(n=200_000, d=64, centers=10, box=5.0, std=(2.0, 2.0), noise=0.0, zero_cols=0,
               eps=[6.0, 9.0, 12.0], min_samples=[10, 50, 200], budget=128 * 10**9, npr=0,
               desc="Dense-route stress as written: N=200,000 D=64, 10 centres U[-5,5]^64, std 2.0, "
                    "no noise; 3x3 grid"),
    # the same points with eps at sampled pair-distance quantiles, so that the largest eps links
    # about 20% of all pairs (the dense regime the stress case is meant to exercise)
    "c5q": dict(n=200_000, d=64, centers=10, box=5.0, std=(2.0, 2.0), noise=0.0, zero_cols=0,
                eps=None, eps_quantiles=(0.05, 0.10, 0.20), min_samples=[10, 50, 200], budget=128 * 10**9,
                npr=0,
                desc="Dense-route stress, calibrated: the C5 points with eps at the 5/10/20% quantiles "
                     "of 200,000 sampled pair distances; 3x3 grid"),
    # the same grid under a 64 GB budget: the whole pair list + CSR (~117 GB for 4e9 neighbour
    # pairs) no longer fits, so the graph is built one row batch at a time
    "c5qb": dict(n=200_000, d=64, centers=10, box=5.0, std=(2.0, 2.0), noise=0.0, zero_cols=0,
                 eps=None, eps_quantiles=(0.05, 0.10, 0.20), min_samples=[10, 50, 200], budget=64 * 10**9,
                 npr=0,
                 desc="Dense-route stress, calibrated, memory-bounded: the c5q grid under a 64 GB budget "
                      "(the graph is built per row batch)"),
}


def calibrated_eps(pts: np.ndarray, quantiles, pairs: int = 200_000, seed: int = 1) -> list[float]:
    """eps values at the given quantiles of the distances of `pairs` random point pairs (i != j),
    as float32 values, ascending."""
    rng = np.random.default_rng(seed)
    n = len(pts)
    i = rng.integers(0, n, size=pairs)
    j = (i + rng.integers(1, n, size=pairs)) % n
    dist = np.sqrt(((pts[i].astype(np.float64) - pts[j].astype(np.float64)) ** 2).sum(axis=1))
    eps = sorted({float(np.float32(v)) for v in np.quantile(dist, list(quantiles))})
    return eps


def workload_eps(cfg: dict, pts: np.ndarray) -> list[float]:
    return list(cfg["eps"]) if cfg.get("eps") else calibrated_eps(pts, cfg["eps_quantiles"])


def make_points(cfg: dict, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    n, d, zc = cfg["n"], cfg["d"], cfg["zero_cols"]
    di = d - zc
    centres = rng.uniform(-cfg["box"], cfg["box"], size=(cfg["centers"], di))
    lo, hi = cfg["std"]
    std = rng.uniform(lo, hi, size=cfg["centers"]) if hi > lo else np.full(cfg["centers"], lo)
    m = n - int(round(cfg["noise"] * n))
    assign = rng.integers(0, cfg["centers"], size=m)
    pts = np.zeros((n, d), dtype=np.float32)
    pts[:m, :di] = (centres[assign] + rng.standard_normal((m, di)) * std[assign, None]).astype(np.float32)
    pts[m:, :di] = rng.uniform(-cfg["box"], cfg["box"], size=(n - m, di)).astype(np.float32)
    return pts


# ---- clocks during the timed region: a separate nvidia-smi process (reads only) ----------------
class ClockSampler:
    """Samples SM clocks and clock-event reasons every 20 ms in a child process (NVML through
    nvidia_ml_py, else nvidia-smi -lms 20), each sample time-stamped; stop() keeps the samples
    that fall inside the marked timed region, so sampling never competes with this process for
    the interpreter lock and a short region still gets samples."""

    CHILD = r"""
import sys, time
import pynvml as N
N.nvmlInit()
hs = [N.nvmlDeviceGetHandleByIndex(int(i)) for i in sys.argv[1].split(",")]
mx = [N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM) for h in hs]
get = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or N.nvmlDeviceGetCurrentClocksThrottleReasons
out = open(sys.argv[2], "w", buffering=1)
while True:
    t = time.time()
    for h, m in zip(hs, mx):
        out.write("%.6f,%d,%d,%d\n" % (t, N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM), m, get(h)))
    time.sleep(0.02)
"""
    # NVML clock-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, devices):
        import tempfile

        self.devices = ",".join(str(int(x)) for x in devices)
        self.proc = None
        self.t0 = self.t1 = None
        self.tmp = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
        self.tmp.close()

    def start(self):
        import subprocess
        import sys as _sys

        try:
            import pynvml  # noqa: F401
            self.proc = subprocess.Popen([_sys.executable, "-c", self.CHILD, self.devices, self.tmp.name],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml-unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.tmp.name) as f:
            for line in f:
                parts = line.strip().split(",")
                if len(parts) == 4:
                    try:
                        rows.append((float(parts[0]), float(parts[1]), float(parts[2]), int(parts[3])))
                    except ValueError:
                        pass
        try:
            os.unlink(self.tmp.name)
        except OSError:
            pass
        t0, t1 = self.t0 or 0.0, self.t1 or time.time()
        inside = [r for r in rows if t0 <= r[0] <= t1]
        reasons = sorted({nm for r in inside for nm, bit in self.BITS.items() if r[3] & bit})
        clocks = [r[1] for r in inside]
        return {"sm_mhz": float(np.median(clocks)) if clocks else None,
                "sm_max_mhz": rows[-1][2] if rows else None, "reasons": reasons,
                "samples_in_timed_region": len(inside), "samples": len(rows),
                "timed_region_s": t1 - t0, "sampler": "NVML every 20 ms in a child process"}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def sgemm_fp32_peak(torch, dev) -> float:
    """Measured CUDA-core FP32 throughput: cuBLAS SGEMM 8192^3 with TF32 off, best of 5
    (TFLOP/s, FMA = 2 flops).  The distance kernel is bound by the same FP32 pipes."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a = torch.randn(8192, 8192, device=dev)
        b = torch.randn(8192, 8192, device=dev)
        torch.matmul(a, b)
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            e1.synchronize()
            best = max(best, 2 * 8192**3 / (e0.elapsed_time(e1) * 1e-3) / 1e12)
        del a, b
        return best
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def index_bits(n: int) -> int:
    """The reference CLI's --index auto: int64 iff N*N >= INT32_MAX (src/main.cu:681-689)."""
    return 64 if n * n >= 2**31 - 1 else 32


def cpu_pipeline(pts: np.ndarray, eps, ms, budget: int, npr: int, target_s: float = 12.0) -> dict:
    """The CPU restatement of the whole path (oracle.fit_multi_stream: per-eps degrees, per-batch
    neighbour lists, weak-CC + merge of every configuration, relabel), on every host core, over
    the first N' points of the workload, N' sized so that one run takes about `target_s`.  The
    grid time extrapolates to N as (N / N')^2: the two distance passes, O(N^2), are nearly all
    of it (the labelling is linear in the graph)."""
    import batching
    import oracle

    threads = oracle.default_threads()
    n, k, l = len(pts), len(eps), len(ms)

    def run(m):
        bs = batching.compute_batch_size(m, k, l, budget, use_cuvs=True, neigh_hint=npr, index_bits=index_bits(m))
        t0 = time.perf_counter()
        oracle.fit_multi_stream(pts[:m], eps, ms, bs, threads)
        return time.perf_counter() - t0, bs

    m = min(n, 4096)
    dt, bs = run(m)
    while dt < target_s / 8 and m < n:
        m = min(n, m * 2)
        dt, bs = run(m)
    m2 = min(n, int(m * (target_s / max(dt, 1e-6)) ** 0.5))
    if m2 > m * 1.2:
        m = m2
        dt, bs = run(m)
    grid_s = dt * (n / m) ** 2
    return {"value": float(n) * n / grid_s, "unit": "pairs/s", "grid_wall_s": grid_s, "cores": threads,
            "kind": "port",
            "sample": f"oracle.fit_multi_stream (distance passes + per-batch lists + weak-CC/merge of all "
                      f"{k * l} configurations + relabel) on the first {m} of {n} points ({dt:.1f} s, "
                      f"batch size {bs}); grid time extrapolated by (N/{m})^2",
            "seconds": dt}


def dv_baseline(pts: np.ndarray, eps, ms, target_s: float = 10.0) -> dict:
    """The reference's own CPU validation DBSCAN (tools/dbscan_validation.py: build_epsilon_graph
    per eps + structure per minPts, dense float64) when the reference's tools are importable (a
    checkout named by DBM_REFERENCE_ROOT, or an install under baseline/_ref), on the first N''
    points, extrapolated by (N/N'')^2 (its dense N x N graph makes the full size infeasible)."""
    roots = [os.environ.get("DBM_REFERENCE_ROOT", ""), str(ROOT / "baseline" / "_ref")]
    dv = None
    for r in roots:
        if r and (Path(r) / "tools" / "dbscan_validation.py").exists():
            sys.path.insert(0, str(Path(r) / "tools"))
            try:
                import dbscan_validation as dv  # noqa: F401
            except Exception:
                dv = None
            finally:
                sys.path.pop(0)
            break
    if dv is None:
        return {"unavailable": "the reference's tools/dbscan_validation.py is not installed here: the reference "
                               "has no setup.py or pyproject.toml, so its offline pip install fails, and its "
                               "checkout is not present on this machine"}
    n = len(pts)

    def run(m):
        t0 = time.perf_counter()
        for e in eps:
            g = dv.build_epsilon_graph(pts[:m].astype(np.float64), float(e), max_n=m)
            for v in ms:
                g.structure(int(v))
        return time.perf_counter() - t0

    m = min(n, 1024)
    dt = run(m)
    while dt < target_s / 4 and m < n:
        m = min(n, m * 2)
        dt = run(m)
    grid_s = dt * (n / m) ** 2
    return {"value": float(n) * n / grid_s, "unit": "pairs/s", "grid_wall_s": grid_s,
            "cores": os.cpu_count(), "kind": "reference (tools/dbscan_validation.py)",
            "sample": f"build_epsilon_graph x {len(eps)} eps + structure x {len(ms)} minPts on the first {m} of {n} "
                      f"points ({dt:.1f} s); grid time extrapolated by (N/{m})^2"}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def e2e_leg(h, pts, eps, ms, kw, labels, flush, steps, ws, dev, torch, dist, pairs):
    """Host buffers through dbm_fit_multi_host: pinned points copied in and labels copied out
    inside every timed step (wall clock around the call)."""
    k, l, n = len(eps), len(ms), len(pts)
    xp = torch.from_numpy(pts).pin_memory()
    lab_host = torch.empty((k * l, n), dtype=torch.int32).pin_memory()
    h.fit_multi(xp.numpy(), eps, ms, labels_out=lab_host.numpy(), **kw)
    e2e_t = []
    for _ in range(steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        h.fit_multi(xp.numpy(), eps, ms, labels_out=lab_host.numpy(), **kw)
        e2e_t.append(time.perf_counter() - t0)
    assert np.array_equal(lab_host.numpy(), labels.cpu().numpy()), "host and device paths disagree"
    e2e_s = float(np.sum(e2e_t))
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    return pairs * ws * steps / e2e_s, e2e_s


def e2e_leg_sharded(one_fit, x, pts, labels, flush, steps, rank, dev, torch, dist, pairs, ws):
    """Sharded e2e through dbscan_multi.parallel.sharded_fit_multi with host points: each rank
    copies its 1/G row slice from pinned memory and the points are all-gathered over NCCL, the
    sharded fit runs, rank 0 copies the gathered labels out; wall clock per step, max over ranks."""
    xp = torch.from_numpy(pts).pin_memory()
    lab_host = torch.empty(tuple(labels.shape), dtype=torch.int32).pin_memory()
    one_fit(xp)
    ts = []
    for _ in range(steps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        one_fit(xp)
        if rank == 0:
            lab_host.copy_(labels, non_blocking=True)
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t0)
    t = torch.tensor([float(np.sum(ts))], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    return pairs * steps / e2e_s, e2e_s


def run_reference(args, cfg) -> None:
    """The reference arm: the CPU restatement of the whole path on the host cores, same metric."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    pts = make_points(cfg)
    cfg["eps"] = workload_eps(cfg, pts)
    ms = cfg["min_samples"]
    cb = None
    values, grids = [], []
    per_step = args.cpu_seconds / max(1, args.steps)
    for _ in range(args.warmup):
        cpu_pipeline(pts, cfg["eps"], ms, cfg["budget"], cfg["npr"], target_s=min(2.0, per_step))
    for _ in range(args.steps):
        cb = cpu_pipeline(pts, cfg["eps"], ms, cfg["budget"], cfg["npr"], target_s=per_step)
        values.append(cb["value"])
        grids.append(cb["grid_wall_s"])
    value = float(np.median(values))
    grid_s = float(np.median(grids))
    n = cfg["n"]
    out = {
        "impl": "reference", "metric": "pair_distances_per_s_effective", "grid_wall_s": grid_s, "value": value,
        "unit": "pairs/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": grid_s * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, "desc": cfg["desc"], "n": n, "d": cfg["d"],
                   "eps": cfg["eps"], "min_samples": ms, "max_bytes_per_batch": cfg["budget"]},
        "cpu_baseline": {"value": value, "unit": "pairs/s", "cores": cb["cores"], "kind": "port",
                         "sample": cb["sample"], "grid_wall_s": grid_s},
        "e2e": {"value": value, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "extrapolated": True,
        "note": "the reference's own path needs RAFT/cuVS/RMM and a GPU and cannot be built offline; its "
                "CPU restatement (oracle/dbm_oracle.c: sequential fp32 FMA distances, literal weak-CC + "
                "merge labelling, every host core) is timed over the whole grid on a subset of the "
                "points and extrapolated to N; ms_per_step is that extrapolated grid time",
    }
    print(json.dumps(out), flush=True)


def screen_roofline(stats, screen_ms, d, n, ws, dms, sm_mhz, args) -> dict:
    """Roofline of dist_screen_kernel: tcgen05 tf32 GEMM work of the screen (128 x 128 x KP per
    screened tile pair, FMA = 2 flops) over the kernel's own event-timed duration, against the
    tf32 dense peak taken as half the measured bf16 GEMM rate."""
    kp = 8 * ((d + 4 + 7) // 8)
    screened = int(stats.get("screened_tile_pairs", 0))
    sms = float(np.mean(screen_ms)) if screen_ms else float("nan")
    flops = float(screened) * 128 * 128 * kp * 2
    achieved = flops / (sms * 1e-3) / 1e12
    mp = measured_peaks()
    bf16 = mp.get("bf16_tflops")
    peak = bf16 / 2 if bf16 else 1590.0 / 2
    cands = int(stats.get("screen_candidates", 0))
    traffic = None
    tp = ROOT / "profiles" / "dist_screen_kernel_traffic.json"
    if tp.exists() and not args.n and ws == 1:
        try:
            traffic = json.loads(tp.read_text()).get(args.config)
        except Exception:
            traffic = None
    pairs_bounded = float(screened) * 128 * 128
    return {
        "bound": "tensor", "kernel": "dist_screen_kernel", "achieved": achieved, "peak": peak,
        "unit": "TFLOP/s", "frac": achieved / peak if peak else None,
        "peak_source": ("tf32 dense = 1/2 of the measured bf16 cuBLAS rate in MEASURED_PEAKS.json" if bf16
                        else "tf32 dense = 1/2 of the fallback bf16 rate"),
        "traffic": traffic, "flops_per_launch": flops, "ms_per_launch": sms,
        "screened_tile_pairs": screened, "pairs_bounded_per_s": pairs_bounded / (sms * 1e-3),
        "candidates": cands, "exact_chain_pairs": cands,
        "exact_chain_flops": float(cands) * 3 * d,
        "fallback_tile_pairs": int(stats.get("fallback_tile_pairs", 0)),
        "tile_pairs_kept": stats.get("tile_pairs_kept"),
        "distance_phase_ms": dms,
        "accounting": ("unit = one screened 128x128 tile pair: 128*128*KP tf32 multiply-adds (KP = D + 4 "
                       "rounded to 8: centred coordinates + the two split bound terms); the kernel also runs "
                       "the exact fp32 chain (3D flops) for every candidate pair, reported separately. The "
                       "tensor fraction is low by design: the kernel is bound by CUDA-core issue of the "
                       "operand build and the screen epilogue, not by the MMA."),
    }


def exact_roofline(stats, unique_pairs, d, dms, sm_mhz, torch, dev, args, ws) -> dict:
    """Roofline of dist_tri_kernel (the exact fp32 tile kernel, used when the screen does not
    apply): flops actually evaluated over the distance phase."""
    flops = unique_pairs * 3.0 * d  # D FSUB + D FFMA (FMA = 2 flops)
    work_frac = float(stats.get("dist_work_fraction", 1.0) or 1.0)
    flops_exec = flops * work_frac
    achieved = flops_exec / (dms * 1e-3) / 1e12
    peak = sgemm_fp32_peak(torch, dev)
    nominal = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
    lane_frac = (unique_pairs * 2.0 * d * work_frac) / (dms * 1e-3) / (148 * 128 * sm_mhz * 1e6)
    traffic = None
    tp = ROOT / "profiles" / "dist_tri_kernel_traffic.json"
    if tp.exists() and not args.n and ws == 1:
        try:
            traffic = json.loads(tp.read_text()).get(args.config)
        except Exception:
            traffic = None
    return {"bound": "fp32", "kernel": "dist_tri_kernel", "achieved": achieved,
            "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak if peak else None,
            "peak_source": "measured here: cuBLAS SGEMM 8192^3, TF32 off (no FP32 figure in MEASURED_PEAKS.json)",
            "peak_nominal": nominal, "fp32_lane_utilisation": lane_frac,
            "flops_per_launch": flops_exec, "ms_per_launch": dms, "executed_fraction": work_frac,
            "full_grid_flops": flops, "attainable_frac": 0.75, "traffic": traffic,
            "accounting": "flops evaluated: unique pairs N(N-1)/2 x 3D flops (D FSUB + D FFMA, FMA = 2) x "
                          "executed_fraction; under this accounting the ceiling is 75% of the FMA-counted peak"}


def label_roofline(nnz_eps, n, l, stats, label_ms, ws) -> dict:
    """HBM roofline of the labelling (per-batch compaction, batched connected components, border
    fold, relabel).  Algorithmic bytes per grid, the CC accounting of one sweep per configuration
    (a column index and a label gather per entry, the labels read and written, the core mask):
    sum over configs of 8 * nnz(eps of the config) + 8 N + N / 8; plus, where the fit compacts the
    smaller-eps slabs (annotated batches of a dense graph, >= 64 entries per row; sparse batches
    read each entry's eps from its code instead), the compaction's 4 bytes read per max-eps entry
    and 8 bytes written per kept smaller-eps entry.  Over the phase's event time (the labelling
    kernels' share of the step)."""
    mp = measured_peaks()
    peak = mp.get("hbm_gbs") or 6650.0
    bytes_cc = sum(l * (8.0 * v + 8.0 * n + n / 8.0) for v in nnz_eps)
    compacts = int(stats.get("annotated_batches", 0) or 0) > 0 and bool(nnz_eps) and nnz_eps[-1] >= 64 * n
    bytes_compact = (4.0 * nnz_eps[-1] + 8.0 * sum(nnz_eps[:-1])) if compacts and len(nnz_eps) > 1 else 0.0
    ms = float(np.mean(label_ms)) if label_ms else float("nan")
    achieved = (bytes_cc + bytes_compact) / (ms * 1e-3) / 1e9 if ms and ms > 0 else None
    return {"bound": "hbm", "kernels": "filter_all (dense annotated batches), cc_touch/union/best/border, "
                                       "cc_root_bits/labels",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak if achieved else None,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if mp.get("hbm_gbs") else "fallback 6650 GB/s",
            "bytes_per_grid": bytes_cc + bytes_compact, "ms_per_grid": ms, "traffic": None,
            "note": "the union-find gathers are latency-bound and mostly L2-resident, so the phase runs far "
                    "below the HBM roofline; on several GPUs this is the rank's own share"
                    + (" (max over ranks not taken)" if ws > 1 else "")}


def label_checks(args, labels, one_fit, h, x, eps, ms, kw, ws, rank, dev, torch, dist) -> dict:
    """One untimed fit, then (N > 1) its labels against a one-GPU fit of the same inputs and
    budget on rank 0, and (full-size workloads) against the oracle's per-configuration SHA-256
    digests.  Flags: 1 match, 0 mismatch, 2 not applicable; combined with MIN over ranks."""
    import hashlib

    one_fit()
    torch.cuda.synchronize()
    flags = torch.full((2,), 2, dtype=torch.int32, device=dev)
    if ws > 1 and rank == 0:
        single = torch.empty_like(labels)
        h.fit_multi(x, eps, ms, labels_out=single, **kw)
        flags[0] = int(torch.equal(single, labels))
    fx_path = ROOT / "tests" / "golden" / "full_size_labels.json"
    if rank == 0 and not args.n and fx_path.exists():
        fx = json.loads(fx_path.read_text()).get(args.config)
        if fx is not None:
            host = labels.cpu().numpy()
            got = [hashlib.sha256(np.ascontiguousarray(r, dtype="<i4").tobytes()).hexdigest() for r in host]
            flags[1] = int(got == [c["sha256"] for c in fx["configs"]])
    if ws > 1:
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    f = [int(v) for v in flags.tolist()]
    out = {}
    if f[0] != 2:
        out["labels_match_1gpu"] = bool(f[0])
    if f[1] != 2:
        out["labels_match_oracle"] = bool(f[1])
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg (profiling runs)")
    ap.add_argument("--n", type=int, default=0, help="override N (small cases for ncu captures)")
    ap.add_argument("--no-clocks", action="store_true", help="diagnostics: time without the clock sampler")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.n:
        cfg["n"] = args.n
        cfg["desc"] += f" [N overridden to {args.n}]"

    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist

    import dbscan_multi as dm

    ws, rank, local = dist_env()
    if ws > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    n, d = cfg["n"], cfg["d"]
    pts = make_points(cfg)
    cfg["eps"] = workload_eps(cfg, pts)
    eps, ms = cfg["eps"], cfg["min_samples"]
    k, l = len(eps), len(ms)
    x = torch.from_numpy(pts).to(dev)
    h = dm.DbscanMulti(local)
    kw = dict(neigh_per_row=cfg["npr"])
    if cfg["budget"]:
        kw["max_bytes_per_batch"] = cfg["budget"]
    labels = torch.empty((k * l, n), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2

    h.set_phase_timing(True)
    if ws > 1:
        from dbscan_multi import parallel

        stages = parallel.DeviceStages(h)
        if "max_bytes_per_batch" not in kw:
            kw["max_bytes_per_batch"] = stages.default_budget()
        # budget and CSR memory cap agreed once (one collective), not in every step
        limits = parallel.agree_limits(stages, kw["max_bytes_per_batch"], 0, device=dev)
        dist_events = []
        orig_shard = stages.distance_shard

        def timed_shard(*a, **k2):
            # events around the distance stage, read after the step (no extra synchronisation)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            out = orig_shard(*a, **k2)
            e1.record(stream)
            dist_events.append((e0, e1))
            return out

        stages.distance_shard = timed_shard

        def one_fit(x_in=None):
            r = parallel.sharded_fit_multi(stages, x if x_in is None else x_in, eps, ms, limits=limits,
                                           device=None if x_in is None else dev, **kw)
            labels.copy_(r.labels)
            e0, e1 = dist_events.pop()
            e1.synchronize()
            dist_events.clear()
            r.stats["ms_distance"] = e0.elapsed_time(e1)
            sh = stages.last_shard_stats
            for key in ("ms_screen", "screened_tile_pairs", "fallback_tile_pairs", "screen_candidates",
                        "tile_pairs_kept", "dist_work_fraction"):
                r.stats[key] = sh.get(key, 0)
            r.stats["launches"] = r.stats.get("launches", 0) + sh.get("launches", 0)
            return r
    else:
        def one_fit():
            return h.fit_multi(x, eps, ms, labels_out=labels, **kw)
    # one sampler for all of this node's GPUs, on rank 0 only (a poller per rank measurably slows
    # the host side of a sharded fit); --no-clocks is for diagnostics only
    clocks = ClockSampler(range(ws) if ws > 1 else [local])
    if rank == 0 and not args.no_clocks:
        clocks.start()
    for _ in range(args.warmup):
        one_fit()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    # correctness before timing: the sharded labels against a one-GPU fit, and the labels against
    # the oracle's digests of this workload (tests/golden/full_size_labels.json, full size only)
    checks = label_checks(args, labels, one_fit, h, x, eps, ms, kw, ws, rank, dev, torch, dist)
    label_ms = []

    times, dist_ms, screen_ms, stats = [], [], [], None
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    clocks.mark_start()
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        r = one_fit()
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
        dist_ms.append(r.stats["ms_distance"])
        label_ms.append((r.stats.get("ms_label") or 0.0) + (r.stats.get("ms_relabel") or 0.0))
        screen_ms.append(r.stats.get("ms_screen", 0.0))
        stats = r.stats
    torch.cuda.synchronize()
    clocks.mark_end()
    if ws > 1:
        dist.barrier()
    clk = clocks.stop()
    # per-eps directed neighbour entries (self pairs excluded), for the labelling roofline
    nnz_eps = [int(v) for v in list(stats.get("nnz_per_eps", []))[:k]]
    total_ms = float(np.sum(times))
    rank_spread = None
    if ws > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t2 = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t2, op=dist.ReduceOp.MIN)
        total_ms = float(t.item())
        rank_spread = [float(t2.item()) / args.steps, total_ms / args.steps]
    ms_per_step = total_ms / args.steps
    pairs = float(n) * float(n)
    value = pairs * (1 if ws > 1 else ws) * args.steps / (total_ms * 1e-3)

    # e2e through the host-buffer entry point: pinned points in, labels out, every step
    h.set_phase_timing(False)
    if args.no_e2e:
        e2e_value, e2e_s = None, None
    elif ws > 1:
        e2e_value, e2e_s = e2e_leg_sharded(one_fit, x, pts, labels, flush, args.steps, rank, dev, torch, dist,
                                           pairs, ws)
    else:
        e2e_value, e2e_s = e2e_leg(h, pts, eps, ms, kw, labels, flush, args.steps, ws, dev, torch, dist,
                                   pairs)
    # roofline of the dominant kernel (this rank's share)
    unique_pairs = n * (n - 1) / 2 / ws
    dms = float(np.mean(dist_ms)) if dist_ms else float("nan")
    sm_mhz = clk.get("sm_mhz") or 1965.0
    screened = int(stats.get("screened_tile_pairs", 0) or 0)
    fallback = int(stats.get("fallback_tile_pairs", 0) or 0)
    if screened > 0 and 2 * fallback <= screened:
        roofline = screen_roofline(stats, screen_ms, d, n, ws, dms, sm_mhz, args)
    else:
        # no screen, or a dense regime where most tile pairs go back to the exact kernel: that
        # kernel dominates; its time is the distance phase less the screen pass
        tri_ms = dms - (float(np.mean(screen_ms)) if screened > 0 and screen_ms else 0.0)
        roofline = exact_roofline(stats, unique_pairs, d, tri_ms, sm_mhz, torch, dev, args, ws)
        if screened > 0:
            roofline["screened_tile_pairs"] = screened
            roofline["fallback_tile_pairs"] = fallback
            roofline["ms_per_launch_note"] = "distance phase minus the screen pass (order, boxes and prune included)"

    if rank == 0:
        cb = None
        if not args.no_cpu_baseline and ws == 1:
            cb = cpu_pipeline(pts, eps, ms, cfg["budget"], cfg["npr"], target_s=args.cpu_seconds)
            cb.pop("seconds", None)
            cb["dv"] = dv_baseline(pts, eps, ms)
        out = {
            "metric": "pair_distances_per_s_effective",
            "grid_wall_s": ms_per_step / 1e3,
            "value": value,
            "unit": "pairs/s",
            "metric_note": "value = N^2 ordered pairs per grid / grid wall time (the reference's pair-distances/s "
                           "unit); it is an effective rate: pruned and screened pairs are resolved without an "
                           "fp32 distance evaluation (see roofline.exact_chain_pairs)",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded numpy generator with the published configuration's shapes)",
            "config": {"workload": args.config, "desc": cfg["desc"], "n": n, "d": d, "eps": eps,
                       "min_samples": ms, "max_bytes_per_batch": cfg["budget"] or 0,
                       "neigh_per_row": cfg["npr"], "batches": stats["batches"],
                       "batch_size": stats["batch_size"], "parallelism": f"tile-pair shards x{ws} (NCCL)" if ws > 1 else "1gpu",
                       "l2": "flushed (256 MB write) between timed steps"},
            "gpu_launches": (int(stats.get("launches", 0)) + (2 if ws > 1 else 0)) * args.steps,
            "clocks": clk,
            "roofline": roofline,
            "e2e": None if e2e_value is None else {
                "value": e2e_value, "unit": "pairs/s",
                # per rank: its 1/G slice of the points in (the rest arrives over NVLink); rank 0
                # copies the labels out
                "h2d_bytes_per_step": int(-(-n // ws) * d * 4), "d2h_bytes_per_step": int(k * l * n * 4),
                "ms_per_step": e2e_s / args.steps * 1e3},
            "graph": {"edges": stats["edges"], "total_nnz_max_eps": stats["total_nnz_max_eps"],
                      "distance_passes": stats["distance_passes"], "nnz_per_eps": nnz_eps,
                      "streamed": bool(stats.get("streamed", 0)),
                      "workspace_bytes": int(stats.get("workspace_bytes", 0) or 0)},
            "roofline_labelling": label_roofline(nnz_eps, n, l, stats, label_ms, ws),
            "rank_ms_per_step_min_max": rank_spread,
            "phase_ms": {"distance": dms, "screen_kernel": float(np.mean(screen_ms)) if screen_ms else None,
                         "graph": stats.get("ms_graph"), "label": stats.get("ms_label"),
                         "relabel": stats.get("ms_relabel")},
            "cpu_baseline": cb,
            "hbm_peak_gbs": measured_peaks().get("hbm_gbs"),
            **checks,
        }
        print(json.dumps(out), flush=True)
    h.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if checks.get("labels_match_1gpu") is False or checks.get("labels_match_oracle") is False:
        sys.exit(1)


if __name__ == "__main__":
    main()
