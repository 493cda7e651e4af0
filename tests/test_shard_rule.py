"""The distance shards' item rule (dbm_internal.cuh shard_item / shard_items) against its Python
mirror (dbscan_multi.parallel.shard_items), on the host: a small program built with nvcc from
the kernels' own header prints each shard's global item indices.  No GPU is needed."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import dbscan_multi.parallel as parallel

CSRC = Path(__file__).resolve().parents[1] / "cuml-dbscanmulti_b200" / "csrc"

PROGRAM = r"""
#include "dbm_internal.cuh"
#include <cstdio>
int main()
{
  const long long totals[] = {0, 1, 63, 64, 65, 200, 4096, 3000001};
  const int worlds[] = {1, 2, 3, 8};
  for (long long t : totals)
    for (int S : worlds)
      for (int s = 0; s < S; ++s) {
        const long long cnt = dbm::shard_items(t, s, S);
        // every valid local item, capped for the large total (first and last 300)
        std::printf("%lld %d %d %lld", t, S, s, cnt);
        for (long long i = 0; i < cnt; ++i) {
          if (cnt > 600 && i == 300) i = cnt - 300;
          std::printf(" %lld:%lld", i, (long long)dbm::shard_item(i, s, S));
        }
        std::printf("\n");
      }
  return 0;
}
"""


@pytest.fixture(scope="module")
def shard_dump(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    d = tmp_path_factory.mktemp("shard_rule")
    src = d / "shard_rule.cu"
    src.write_text(PROGRAM)
    exe = d / "shard_rule"
    subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{CSRC}",
                    "-o", str(exe), str(src)], check=True, capture_output=True)
    return subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines()


def test_device_rule_equals_the_python_mirror(shard_dump):
    assert shard_dump
    for line in shard_dump:
        t, S, s, cnt = (int(v) for v in line.split()[:4])
        want = parallel.shard_items(t, s, S)
        assert cnt == len(want), line[:80]
        for p in line.split()[4:]:
            i, g = (int(v) for v in p.split(":"))
            assert want[i] == g


def test_shards_cover_every_item_once(shard_dump):
    seen: dict[tuple[int, int], int] = {}
    for line in shard_dump:
        t, S, s, cnt = (int(v) for v in line.split()[:4])
        seen[(t, S)] = seen.get((t, S), 0) + cnt
    for (t, S), total in seen.items():
        assert total == t
    # and the Python mirror is a partition for the small totals
    for t in (0, 1, 63, 64, 65, 200, 4096):
        for S in (1, 2, 3, 8):
            allg = np.sort(np.concatenate([parallel.shard_items(t, s, S) for s in range(S)]))
            assert np.array_equal(allg, np.arange(t))
