"""CPU emulation of the tensor-core screen's bound (dist_tc.cu), checked on near-boundary pairs.

The screened distance pass discards a pair when V = a_i.a_j - h_i - g_j, computed by a tf32
tcgen05 GEMM, has its sign bit set.  Correctness of every label rests on one inequality: for a
pair whose reference chain (src/multi/eps_neighborhood.cuh:151-158) gives acc <= E = eps2_max,
V > 0.  This file restates the kernel's arithmetic in numpy as the kernel source states it:

* a_p = tf32_rn(fl32(x_p - c)) per coordinate (round to nearest, ties away, on the bit pattern);
* n_i (and m_j): fp32 sums of squares in four interleaved partial sums, then (n0+n1)+(n2+n3);
* h_i, g_j: the kernel's directed-rounding formulas (row_slack / col_slack / norm_slack);
* -h and -g split into two tf32 terms each (put_ext);
* the tensor core's fp32 accumulation: NOT emulated bit for bit (its order is the hardware's);
  instead the exact sum S of all K products (float64: tf32 x tf32 products are exact) is taken
  at its worst case S - K 2^-22 T, T the sum of the products' magnitudes -- the error model the
  kernel's margins are sized for.

The cases put both tiles' points far from the box centre (|a| up to 200x the search radius),
where the per-row slack is largest, at the K values of the real instances (D = 33: K = 40,
D = 64: K = 72, and a small D).  Every true neighbour, and every pair up to 2^-20 beyond the
boundary, must keep V > 0 under the worst-case accumulation error; the kernel's comment claims
the 2^-13 margins exceed the rounding errors five times over, which is checked too.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

RHO = np.float32(0.00049)
F32 = np.float32


def tf32_rn(v: np.ndarray) -> np.ndarray:
    """dist_tc.cu tf32_rn: (bits + 0x1000) & 0xFFFFE000."""
    b = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)
    return ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


def round_up(x64: np.ndarray) -> np.ndarray:
    """float64 value -> the smallest float32 >= it (exact when x64 is the exact result)."""
    f = np.asarray(x64, dtype=np.float64).astype(np.float32)
    low = f.astype(np.float64) < x64
    return np.where(low, np.nextafter(f, np.float32(np.inf)), f).astype(np.float32)


def round_down(x64: np.ndarray) -> np.ndarray:
    f = np.asarray(x64, dtype=np.float64).astype(np.float32)
    high = f.astype(np.float64) > x64
    return np.where(high, np.nextafter(f, np.float32(-np.inf)), f).astype(np.float32)


def mul_ru(a, b):
    return round_up(np.asarray(a, np.float64) * np.asarray(b, np.float64))


def add_ru(a, b):
    return round_up(np.asarray(a, np.float64) + np.asarray(b, np.float64))


def sub_rd(a, b):
    return round_down(np.asarray(a, np.float64) - np.asarray(b, np.float64))


def sqrt_ru(a):
    return round_up(np.sqrt(np.asarray(a, np.float64)))


def norm_slack(n, se):
    r = sqrt_ru(mul_ru(n, F32(1.0000153)))
    return mul_ru(mul_ru(F32(2.0) * RHO, r), add_ru(se, mul_ru(RHO, r)))


def row_slack(n, se):
    s2 = mul_ru(se, se)
    h = F32(0.5) * sub_rd(sub_rd(n, s2), norm_slack(n, se))
    return sub_rd(h, mul_ru(F32(0.0001220703125), add_ru(n, s2)))


def col_slack(m, se):
    g = F32(0.5) * sub_rd(m, norm_slack(m, se))
    return sub_rd(g, mul_ru(F32(0.0001220703125), m))


def sqrt_e(eps2: np.float32, d: int) -> np.float32:
    """Host side of launch_screened_distance: s = sqrt(E (1 + (D+3) 2^-24)) rounded up."""
    e = float(eps2) * (1.0 + (d + 3) * math.ldexp(1.0, -24))
    sq = np.float32(math.sqrt(e))
    while float(sq) * float(sq) < e:
        sq = np.nextafter(sq, np.float32(np.inf))
    return np.float32(sq)


def squared_norm(w: np.ndarray) -> np.ndarray:
    """build_row: four partial fp32 sums over t = 4*ch + h (w tf32, so w*w is exact in fp32 and
    each fma is one fp32 rounding of an exact sum), then (n0 + n1) + (n2 + n3)."""
    kp = w.shape[1]
    nq = np.zeros((w.shape[0], 4), np.float32)
    for t in range(kp):
        nq[:, t % 4] = (nq[:, t % 4] + w[:, t] * w[:, t]).astype(np.float32)
    return ((nq[:, 0] + nq[:, 1]) + (nq[:, 2] + nq[:, 3])).astype(np.float32)


def split(v: np.ndarray):
    """put_ext: -v ~ t1 + t2, both tf32."""
    t1 = tf32_rn((-v).astype(np.float32))
    t2 = tf32_rn(((-v).astype(np.float32) - t1).astype(np.float32))
    return t1, t2


def fp32_chain(xi: np.ndarray, xj: np.ndarray) -> np.ndarray:
    """The reference's acc, emulated in float64 (exact squares; an add may differ from the fp32
    fma by an ulp, far inside the 2^-20 band the test covers)."""
    acc = np.zeros(xi.shape[0], np.float32)
    for t in range(xi.shape[1]):
        diff = (xi[:, t] - xj[:, t]).astype(np.float32)
        acc = (diff.astype(np.float64) ** 2 + acc.astype(np.float64)).astype(np.float32)
    return acc


def screen_values(xi, xj, c, eps2, d):
    """(S, T): the exact K-term sum of the screen's GEMM for each pair and the sum of the
    magnitudes of its terms."""
    kp = 8 * ((d + 4 + 7) // 8)
    se = sqrt_e(eps2, d)
    ai = tf32_rn((xi - c).astype(np.float32))
    aj = tf32_rn((xj - c).astype(np.float32))
    pad = np.zeros((xi.shape[0], kp - d), np.float32)
    ni = squared_norm(np.hstack([ai, pad]))
    mj = squared_norm(np.hstack([aj, pad]))
    h = row_slack(ni, se)
    g = col_slack(mj, se)
    h1, h2 = split(h)
    g1, g2 = split(g)
    prods = ai.astype(np.float64) * aj.astype(np.float64)
    terms = np.hstack([prods, np.stack([h1, h2, g1, g2], axis=1).astype(np.float64)])
    return terms.sum(axis=1), np.abs(terms).sum(axis=1), kp


def near_boundary_pairs(rng, m, d, eps, far):
    """m pairs at distance eps * (1 +- 2^-16 .. 2^-6) in random directions, their first point at
    a random place up to `far` * eps from the tile centre (the origin here; the centre's own
    value cancels in the difference, so placing it at 0 loses nothing)."""
    u = rng.standard_normal((m, d))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    v = rng.standard_normal((m, d))
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    xi = (v * rng.uniform(0, far, (m, 1)) * eps).astype(np.float32)
    rel = rng.choice([-1.0, 1.0], m) * np.exp2(-rng.uniform(6, 16, m))
    xj = (xi + u * (eps * (1.0 + rel))[:, None]).astype(np.float32)
    return xi, xj


@pytest.mark.parametrize("d,eps,far", [(33, 4.5, 200.0), (64, 12.0, 200.0), (33, 4.5, 3.0),
                                       (64, 0.7, 50.0), (5, 0.05, 1000.0)])
def test_every_near_boundary_neighbour_passes_the_screen(d, eps, far):
    rng = np.random.default_rng(d * 1000 + int(far))
    eps2 = np.float32(np.float32(eps) * np.float32(eps))
    c = np.zeros(d, np.float32)
    m_total, checked = 2_100_000, 0
    worst_ratio = np.inf
    while checked < m_total:
        m = 300_000
        xi, xj = near_boundary_pairs(rng, m, d, eps, far)
        acc = fp32_chain(xi, xj)
        keep = acc.astype(np.float64) <= float(eps2) * (1.0 + 2.0**-20)
        S, T, kp = screen_values(xi[keep], xj[keep], c, eps2, d)
        err = kp * 2.0**-22 * T  # worst-case fp32 accumulation of the K products
        assert np.all(S - err > 0), "a near-boundary neighbour fails the screen"
        worst_ratio = min(worst_ratio, float(np.min(S / err)))
        checked += m
    # the margins are sized to exceed the accumulation error five times over
    assert worst_ratio > 5.0, worst_ratio


def test_screen_emulation_rejects_far_pairs():
    """Sanity of the emulation itself: pairs at 3x the radius have V < 0 by a wide margin (the
    screen is not vacuous), and the tf32 rounding is to nearest on 10 mantissa bits."""
    rng = np.random.default_rng(5)
    d, eps = 33, 4.5
    eps2 = np.float32(np.float32(eps) * np.float32(eps))
    u = rng.standard_normal((1000, d))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    xi = rng.uniform(-20, 20, (1000, d)).astype(np.float32)
    xj = (xi + 3 * eps * u).astype(np.float32)
    S, T, kp = screen_values(xi, xj, np.zeros(d, np.float32), eps2, d)
    assert np.all(S + kp * 2.0**-22 * T < 0)
    v = np.array([1.0 + 2.0**-11, 1.0 + 2.0**-11 + 2.0**-20, 1.0 + 3 * 2.0**-11], np.float32)
    assert list(tf32_rn(v)) == [np.float32(1.0 + 2.0**-10), np.float32(1.0 + 2.0**-10),
                                np.float32(1.0 + 2.0**-9)]
