"""Restatement of the reference's batch sizing and batch-correction rules.

TEST INFRASTRUCTURE ONLY (the product implements the same rules natively in
cuml-dbscanmulti_b200/csrc/plan.cpp; tests compare the two).

Reference: src/multi/runner_multi.cuh
  est_mem_per_row_multi      :79-105
  est_mem_fixed_multi        :113-119
  csr_bytes_por_entrada      :214-220
  csr_do_lote_cabe           :222-233
  grau_medido                :236-242
  linhas_de_csr_que_cabem    :256-268
  max_bytes_for_batch_size   :437-447
  compute_batch_size_multi   :458-499
  fit_multi retry loop       :1340-1456
"""

from __future__ import annotations

import math

INT32_MAX = 2**31 - 1
INT64_MAX = 2**63 - 1


def index_bytes(index_bits: int) -> int:
    return 8 if index_bits == 64 else 4


def mem_per_row(n: int, k: int, use_cuvs: bool, neigh_hint: int, isz: int) -> int:
    npr = neigh_hint if neigh_hint > 0 else n
    if use_cuvs:
        per_entry = (2 if k > 1 else 1) * isz + (1 if k > 1 else 0)
        return n + npr * per_entry + 2 * isz + k * isz
    return n + n + (npr + 2) * isz + k * isz


def mem_fixed(n: int, k: int, l: int, isz: int) -> int:
    return n * k * l + n * isz * 2


def max_bytes_for_batch_size(n, k, l, batch_size, use_cuvs=False, neigh_hint=0, index_bits=32):
    isz = index_bytes(index_bits)
    return mem_fixed(n, k, l, isz) + batch_size * mem_per_row(n, k, use_cuvs, neigh_hint, isz) + 1


def compute_batch_size(n, k, l, max_bytes, use_cuvs=False, neigh_hint=0, index_bits=32):
    isz = index_bytes(index_bits)
    per_row = mem_per_row(n, k, use_cuvs, neigh_hint, isz)
    fixed = mem_fixed(n, k, l, isz)
    if not max_bytes > fixed:
        raise ValueError("fixed buffers do not fit")
    bs = (max_bytes - fixed) // per_row
    bs = min(n, bs)
    bs = max(bs, 1)
    imax = INT64_MAX if index_bits == 64 else INT32_MAX
    cap = (imax - 1) // n
    if cap < 1:
        raise ValueError("index type too small for one row")
    return min(bs, cap)


def csr_bytes_per_entry(k: int, use_cuvs: bool, isz: int) -> int:
    if use_cuvs and k > 1:
        return 2 * isz + 1
    return isz


def csr_fits(nnz: int, per_entry: int, available: int) -> bool:
    return 1.1 * float(nnz) * float(per_entry) <= float(available)


def measured_degree(nnz: int, rows: int) -> int:
    return max(1, (nnz + rows - 1) // rows)


def csr_rows_that_fit(degree: int, per_entry: int, available: int) -> int:
    per_row = degree * per_entry
    fit = int(0.8 * available) // max(1, per_row)
    return max(1, fit)


def plan(n, k, l, max_bytes, deg_max, deg_all, use_cuvs, neigh_hint, index_bits, available):
    """Final (batch_size, attempts, corrections) after the reference's retry loop.

    deg_max: per-row degree at the largest eps (len n); deg_all: (k, n) per-eps degrees.
    available: bytes the CSR check compares against (test cap, or free device memory).
    """
    isz = index_bytes(index_bits)
    cap_rows = n
    corrections = 0
    pref_max = [0]
    for v in deg_max:
        pref_max.append(pref_max[-1] + int(v))
    pref_all = []
    for e in range(k):
        p = [0]
        for v in deg_all[e]:
            p.append(p[-1] + int(v))
        pref_all.append(p)
    for attempt in range(3):
        bs = min(compute_batch_size(n, k, l, max_bytes, use_cuvs, neigh_hint, index_bits), cap_rows)
        nb = (n + bs - 1) // bs
        per_entry = csr_bytes_per_entry(k, use_cuvs, isz)
        measured = 0
        if use_cuvs:
            # pass 1 runs batches in reverse and stops at the first that does not fit
            for b in range(nb - 1, -1, -1):
                s, t = b * bs, min(n, (b + 1) * bs)
                nnz = pref_max[t] - pref_max[s]
                if not csr_fits(nnz, per_entry, available):
                    measured = measured_degree(nnz, t - s)
                    break
        else:
            mx = 0
            for b in range(nb):
                s, t = b * bs, min(n, (b + 1) * bs)
                for e in range(k):
                    mx = max(mx, pref_all[e][t] - pref_all[e][s])
            if not csr_fits(mx, per_entry, available):
                measured = measured_degree(mx, bs)
        if measured == 0:
            return bs, attempt + 1, corrections
        corrections += 1
        degree = measured if attempt == 0 else n
        new_cap = csr_rows_that_fit(degree, per_entry, available)
        if not new_cap < bs:
            raise ValueError("CSR does not fit even after shrinking the batch")
        cap_rows = new_cap
    raise ValueError("could not size the batch in 3 attempts")
