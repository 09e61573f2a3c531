"""Host-side rules of bench.py that every line relies on: the rotating input sets of each
workload together exceed the 126 MB L2 twice over (no step finds its inputs left in L2 by
the steps before it), an explicit KTA_BENCH_SETS wins (small ncu captures), and the shards of
the N-column split cover the columns exactly once at every world size."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


class _One:
    world, rank = 1, 0


def _set_bytes(wl) -> float:
    return float(wl.bytes)


@pytest.mark.parametrize("name", ["gemm_f16_1024", "moe_gemm_f16", "w4gemm_f16",
                                  "nvfp4gemm_f16", "gemm_bf16_8192"])
def test_rotating_sets_exceed_twice_the_l2(monkeypatch, name):
    monkeypatch.delenv("KTA_BENCH_SETS", raising=False)
    import bench

    wl = bench.WORKLOADS[name](_One())
    assert wl.nsets >= 4
    assert wl.nsets * _set_bytes(wl) >= 2 * bench.L2_BYTES


def test_explicit_set_count_wins(monkeypatch):
    import bench

    monkeypatch.setenv("KTA_BENCH_SETS", "1")
    monkeypatch.setattr(bench, "NSETS", 1)
    assert bench.sets_for(1e6) == 1


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_column_shards_cover_once(world):
    import bench

    n, align = 7168, 128
    cols = []
    for r in range(world):
        lo, hi = bench.shard(n, world, r, align)
        assert lo % align == 0
        cols.extend(range(lo, hi))
    assert cols == list(range(n))
