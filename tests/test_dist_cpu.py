"""Multi-rank host logic of bench.py on CPU: world_size 2 over gloo (127.0.0.1). Each
rank derives its shard of the GEMM's N columns, its attention (batch, head) pairs and its
decode sequences by LPT with no communication; together the shards cover the work exactly once; the max / sum reductions
over ranks (the bench's timing and throughput) agree on every rank; a rank that raises is
reported on the host and the others end with an error instead of hanging."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out: dict, fail_rank: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench

    d = bench.Dist(world, backend="gloo")
    d.init()
    try:
        if rank == fail_rank:
            raise RuntimeError("planted failure on the host")
        lo, hi = bench.shard(8192, world, rank, align=128)
        dec = bench.DecodeWorkload(d)
        att = bench.AttnWorkload(d)
        d.barrier()
        mx = d.max(float(rank + 1))
        sm = d.sum(float(hi - lo))
        out[rank] = {"cols": (lo, hi), "seqs": sorted(dec.lengths), "tokens": dec.tokens,
                     "max": mx, "sum": sm,
                     "attn": (att.pair_lo, att.pair_hi, att.b, att.hh, att.flops)}
    finally:
        d.close()


def _run(world: int, fail_rank: int = -1) -> tuple[dict, list[int]]:
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode if p.exitcode is not None else -999 for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    return dict(out), codes


def test_two_ranks_shard_without_collective_and_reduce_timings():
    out, codes = _run(2)
    assert codes == [0, 0], codes
    assert out[0]["cols"] == (0, 4096) and out[1]["cols"] == (4096, 8192)
    assert out[0]["max"] == out[1]["max"] == 2.0
    assert out[0]["sum"] == out[1]["sum"] == 8192.0
    sys.path.insert(0, str(ROOT))
    import bench
    import numpy as np

    all_len = sorted(int(x) for x in np.random.default_rng(0).integers(1024, 8193, size=64))
    assert sorted(out[0]["seqs"] + out[1]["seqs"]) == all_len
    t0, t1 = out[0]["tokens"], out[1]["tokens"]
    assert abs(t0 - t1) <= 8192  # LPT balance within one sequence
    assert bench.lpt([5, 4, 3, 3], 2) in ([[0, 3], [1, 2]], [[1, 2], [0, 3]])
    # attention: (batch, head) pairs split into whole batch entries, together every pair once,
    # equal causal work on both ranks
    (lo0, hi0, b0, h0, f0), (lo1, hi1, b1, h1, f1) = out[0]["attn"], out[1]["attn"]
    assert (lo0, hi0, lo1, hi1) == (0, 128, 128, 256)
    assert (b0, h0) == (b1, h1) == (4, 32)
    full = bench.AttnWorkload(bench.Dist(1, backend="gloo"))
    assert f0 == f1 and f0 + f1 == full.flops


@pytest.mark.timeout(300)
def test_a_failing_rank_does_not_hang_the_others():
    _, codes = _run(2, fail_rank=1)
    assert codes[1] != 0
    assert all(c != -999 for c in codes)  # every process ended by itself
