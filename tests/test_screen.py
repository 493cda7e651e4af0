"""The tensor-core screened distance pass (dist_tc.cu) against the exact tile kernel and the oracle.

The screen only decides which pairs the exact fp32 chain re-evaluates, so every mode must give
the same labels, core masks and neighbour-pair count as the exact kernel and the oracle, in
every regime the screen handles differently: sparse (few candidates), dense (candidate queue
overflow -> exact tile kernel), coordinates too large for the bound (-> exact tile kernel),
D from 1 to 64, duplicate points, and the diagonal tile pairs.
"""

from __future__ import annotations

import numpy as np
import pytest

import dbscan_multi as dm
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch

    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def handles(torch_mod):
    hs = {m: dm.DbscanMulti(0) for m in ("auto", "exact", "screened")}
    for m, h in hs.items():
        h.set_distance_mode(m)
    yield hs
    for h in hs.values():
        h.close()


def fit(h, torch, pts, eps, ms, **kw):
    x = torch.from_numpy(np.ascontiguousarray(pts, dtype=np.float32)).to("cuda:0")
    r = h.fit_multi(x, eps, ms, return_core=True, **kw)
    return r.labels.cpu().numpy(), r.core.cpu().numpy().astype(bool), r.stats


def blobs(seed, n, d, centers, std, noise, box, zero_cols=0):
    rng = np.random.default_rng(seed)
    di = d - zero_cols
    c = rng.uniform(-box, box, size=(centers, di))
    m = n - int(noise * n)
    pts = np.zeros((n, d), np.float32)
    a = rng.integers(0, centers, m)
    pts[:m, :di] = c[a] + rng.normal(0, std, (m, di))
    pts[m:, :di] = rng.uniform(-box, box, (n - m, di))
    return pts


CASES = {
    # name: (points, eps, min_samples)
    "c4_like_d33": (blobs(1, 12000, 33, 12, 1.1, 0.05, 20, zero_cols=1), [3.0, 3.5, 4.0, 4.5], [5, 10, 20, 40]),
    "d2_blobs": (blobs(2, 9000, 2, 8, 0.5, 0.05, 10), [0.05, 0.1, 0.2], [5, 10, 20]),
    "d8_c2_like": (blobs(3, 10000, 8, 20, 0.7, 0.05, 10), [0.4, 0.8, 1.2], [10]),
    "d1_line": (blobs(4, 6000, 1, 5, 0.3, 0.1, 10), [0.001, 0.01], [3, 8]),
    "d64_wide": (blobs(5, 8000, 64, 10, 2.0, 0.0, 5), [6.0, 9.0, 12.0], [10, 50, 200]),
    "d17_odd": (blobs(6, 7000, 17, 6, 0.4, 0.1, 3), [0.8, 1.2, 1.6, 2.0], [4, 16]),
    "duplicates": (np.repeat(blobs(7, 2500, 5, 4, 0.2, 0.1, 4), 2, axis=0), [0.0001, 0.2, 0.4], [2, 3, 6]),
    "dense_regime": (blobs(8, 6000, 3, 2, 1.0, 0.0, 1), [1.5, 3.0], [50, 400]),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_screened_equals_exact_and_oracle(handles, torch_mod, name):
    pts, eps, ms = CASES[name]
    want, want_core, _ = oracle.fit_multi(pts, eps, ms)
    lab_x, core_x, st_x = fit(handles["exact"], torch_mod, pts, eps, ms)
    lab_s, core_s, st_s = fit(handles["screened"], torch_mod, pts, eps, ms)
    lab_a, _, _ = fit(handles["auto"], torch_mod, pts, eps, ms)
    assert np.array_equal(lab_x, want) and np.array_equal(core_x, want_core)
    assert np.array_equal(lab_s, want) and np.array_equal(core_s, want_core)
    assert np.array_equal(lab_a, want)
    assert st_s["edges"] == st_x["edges"]
    assert st_x["screened_tile_pairs"] == 0
    assert st_s["screened_tile_pairs"] + st_s["fallback_tile_pairs"] > 0


def test_sparse_case_is_mostly_screened(handles, torch_mod):
    pts, eps, ms = CASES["c4_like_d33"]
    _, _, st = fit(handles["screened"], torch_mod, pts, eps, ms)
    assert st["screened_tile_pairs"] > 0
    assert st["fallback_tile_pairs"] <= st["screened_tile_pairs"] // 10
    # the bound is tight: candidates stay within a small factor of the true neighbour pairs
    assert st["edges"] <= st["screen_candidates"] <= 8 * st["edges"] + 16384


def test_dense_regime_falls_back_to_exact_tiles(handles, torch_mod):
    pts, eps, ms = CASES["dense_regime"]
    _, _, st = fit(handles["screened"], torch_mod, pts, eps, ms)
    assert st["fallback_tile_pairs"] > 0


def test_huge_coordinates_fall_back(handles, torch_mod):
    """Coordinates whose squares overflow float32 cannot be bounded: those tile pairs go to the
    exact kernel, and labels (computed with the same overflowing fp32 chain) still match."""
    rng = np.random.default_rng(11)
    pts = blobs(9, 5000, 4, 5, 0.5, 0.1, 5)
    pts[:200] *= np.float32(3e18)
    eps, ms = [0.3, 0.6], [3, 7]
    want, want_core, _ = oracle.fit_multi(pts, eps, ms)
    lab, core, st = fit(handles["screened"], torch_mod, pts, eps, ms)
    assert np.array_equal(lab, want) and np.array_equal(core, want_core)
    assert st["fallback_tile_pairs"] > 0


@pytest.mark.parametrize("rows", [None, 1000])
def test_screen_with_batches_and_routes(handles, torch_mod, rows):
    import batching

    pts, eps, ms = CASES["c4_like_d33"]
    n = len(pts)
    kw = {}
    bs = None
    if rows:
        kw["max_bytes_per_batch"] = batching.max_bytes_for_batch_size(n, len(eps), len(ms), rows, True, 0, 32)
        bs = batching.compute_batch_size(n, len(eps), len(ms), kw["max_bytes_per_batch"], True, 0, 32)
    want, _, _ = oracle.fit_multi(pts, eps, ms, bs)
    for route in ("annotated", "dense"):
        lab, _, _ = fit(handles["screened"], torch_mod, pts, eps, ms, route=route, index="int32", **kw)
        assert np.array_equal(lab, want)


def test_screened_mode_needs_the_ordering(handles, torch_mod):
    pts = blobs(10, 1000, 3, 3, 0.3, 0.0, 3)
    with pytest.raises(dm.DbmError):
        fit(handles["screened"], torch_mod, pts, [0.2], [4])
    want, _, _ = oracle.fit_multi(pts, [0.2], [4])
    lab, _, _ = fit(handles["auto"], torch_mod, pts, [0.2], [4])
    assert np.array_equal(lab, want)


def test_large_case_screened_equals_exact(handles, torch_mod):
    """C4's distribution at 300k points: labels and neighbour counts equal between the screened
    pass and the exact tile kernel (no oracle at this size)."""
    pts = blobs(12, 300_000, 33, 30, 1.1, 0.05, 20, zero_cols=1)
    eps, ms = [3.0, 3.5, 4.0, 4.5], [5, 10, 20, 40]
    lab_x, core_x, st_x = fit(handles["exact"], torch_mod, pts, eps, ms)
    lab_s, core_s, st_s = fit(handles["screened"], torch_mod, pts, eps, ms)
    assert st_s["edges"] == st_x["edges"] > 0
    assert np.array_equal(lab_s, lab_x) and np.array_equal(core_s, core_x)


# ---- pairs planted exactly at the eps boundary, far from the tile centres ------------------------
def plant_partners(rng, base, e2, offset):
    """For each row x_i of `base` a partner x_j whose reference chain value (fp32 sequential fma,
    src/multi/eps_neighborhood.cuh:151-158) is exactly the float `offset` ulps from e2
    (0: acc == fl(eps^2), the closed ball's edge; +1: the next float above, not a neighbour;
    -1: the float below).  The leading D-1 coordinates carry ~3/4 of the distance in a random
    direction; the last coordinate (kept near 0 in `base`, so its float grid is fine) is scanned
    over consecutive floats until the chain lands on the target.  Returns (partners, ok mask)."""
    m, d = base.shape
    target = np.float32(e2)
    for _ in range(abs(offset)):
        target = np.nextafter(target, np.float32(np.inf if offset > 0 else -np.inf))
    u = rng.standard_normal((m, d - 1))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    part = base.copy()
    part[:, : d - 1] = (base[:, : d - 1] - u * np.sqrt(0.75 * float(e2))).astype(np.float32)
    prefix = oracle.pair_chain(base[:, : d - 1], part[:, : d - 1]).astype(np.float64)
    d_last = np.sqrt(np.maximum(float(target) - prefix, 0.0))
    v0 = (base[:, d - 1] - d_last).astype(np.float32)  # negative: base's last coordinate is in [0, 1)
    steps = np.arange(-3000, 3001, dtype=np.int64)
    ok = np.zeros(m, bool)
    for r in range(m):
        bits = v0[r:r + 1].view(np.int32).astype(np.int64) + steps
        cand = bits.astype(np.int32).view(np.float32)
        trial = np.repeat(part[r:r + 1], len(cand), axis=0)
        trial[:, d - 1] = cand
        acc = oracle.pair_chain(np.repeat(base[r:r + 1], len(cand), axis=0), trial)
        hit = np.flatnonzero(acc == target)
        if hit.size:
            part[r, d - 1] = cand[hit[hit.size // 2]]
            ok[r] = True
    return part, ok


@pytest.mark.parametrize("d,eps", [(33, [4.0, 4.5]), (64, [9.0, 12.0])])
def test_screen_keeps_pairs_planted_at_the_eps_boundary(handles, torch_mod, d, eps):
    """KP = 40 (D = 33) and 72 (D = 64) tf32 columns, the accumulation lengths of the real
    instances.  Base points are spread over [-1000, 1000] in every leading dim, so each tile's
    box centre sits ~1000 sqrt(D) from its points (the per-row slack of the bound is largest
    there, r / s ~ 10^3); partners sit at exactly fl(eps_max^2), one ulp inside and one ulp
    outside.  Degrees and labels of the screened pass must equal the oracle's, every planted
    boundary pair must be found, and no tile pair may fall back to the exact kernel (the
    screen, not the fallback, decided them)."""
    rng = np.random.default_rng(d)
    nb, per = 5000, 300
    base = rng.uniform(-1000, 1000, (nb, d)).astype(np.float32)
    base[:, d - 1] = rng.uniform(0, 1, nb).astype(np.float32)
    e2 = np.float32(np.float32(eps[-1]) * np.float32(eps[-1]))
    parts, oks = [], []
    for v, off in enumerate((0, -1, 1)):
        p, ok = plant_partners(rng, base[v * per:(v + 1) * per], e2, off)
        parts.append(p)
        oks.append(ok)
    assert all(ok.mean() > 0.9 for ok in oks), [ok.mean() for ok in oks]
    pts = np.vstack([base] + parts)
    # planted chain values, re-checked with the oracle's own chain
    for v, off in enumerate((0, -1, 1)):
        acc = oracle.pair_chain(base[v * per:(v + 1) * per][oks[v]], parts[v][oks[v]])
        assert np.all((acc == e2) if off == 0 else ((acc < e2) if off < 0 else (acc > e2)))
    ms = [2, 3]
    want, want_core, want_deg = oracle.fit_multi(pts, eps, ms)
    x = torch_mod.from_numpy(pts).cuda()
    deg = handles["screened"].neighbor_counts(x, eps).cpu().numpy()
    assert np.array_equal(deg, want_deg)
    lab, core, st = fit(handles["screened"], torch_mod, pts, eps, ms)
    assert np.array_equal(lab, want) and np.array_equal(core, want_core)
    assert st["screened_tile_pairs"] > 0 and st["fallback_tile_pairs"] == 0
    # the boundary pairs themselves: in, in, out
    for v, off in enumerate((0, -1, 1)):
        i = np.arange(v * per, (v + 1) * per)[oks[v]]
        j = nb + v * per + np.flatnonzero(oks[v])
        same = lab[-2][i] == lab[-2][j]  # minPts 2 at the largest eps: a planted pair is one cluster
        assert np.all(same & (lab[-2][i] >= 0)) if off <= 0 else np.all(lab[-2][i] == -1)
