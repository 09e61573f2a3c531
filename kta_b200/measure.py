"""Measurement protocol and statistics of a kernel case (the reference's `time` mode).

- ``MeasureParams`` carries the fields and defaults of the reference's protocol record
  (src/kta/measure/protocol.py:27-45): CUDA events per iteration, a 2 x L2 flush before each
  iteration, >= 4 rotating input sets, NaN-filled outputs, warm-up max(10 iterations, 50 ms),
  measured max(100 iterations, 200 ms), median with a 95 % bootstrap CI of 1000 resamples.
- ``bootstrap_median`` / ``significance`` restate src/kta/measure/stats.py:16-61.
- ``time_launches`` runs the timing loop of src/kta/measure/bench.py:124-192 around any
  launch: per iteration refill outputs with NaN, write the flush buffer, then time the single
  launch between two CUDA events; ``time_case`` applies it to a libkta_b200 entry on host
  input sets (rotated per iteration), as the reference's `time` mode does.
"""

from __future__ import annotations

import random
import time
from dataclasses import asdict, dataclass
from typing import Any

import numpy as np


@dataclass(frozen=True)
class MeasureParams:
    timing: str = "cuda_events_per_iteration"
    l2_flush_factor: float = 2.0
    min_input_sets: int = 4
    nan_fill: bool = True
    warmup_min_iters: int = 10
    warmup_min_ms: float = 50.0
    min_iters: int = 100
    min_ms: float = 200.0
    max_iters: int = 100_000
    statistic: str = "median"
    ci_level: float = 0.95
    bootstrap_resamples: int = 1000
    noise_floor_rel: float = 0.011
    significance_factor: float = 3.0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> MeasureParams:
        unknown = set(data) - set(cls.__dataclass_fields__)
        if unknown:
            raise ValueError(f"unknown measurement protocol parameters: {sorted(unknown)}")
        return cls(**data)


V1 = MeasureParams()


def _generator(rng: random.Random) -> np.random.Generator:
    return np.random.default_rng(rng.getrandbits(63))


def bootstrap_median(values: list[float], resamples: int, level: float,
                     rng: random.Random) -> tuple[float, float, float]:
    x = np.asarray(values, dtype=np.float64)
    if x.size == 0:
        raise ValueError("no samples")
    idx = _generator(rng).integers(0, x.size, size=(resamples, x.size))
    meds = np.median(x[idx], axis=1)
    lo, hi = np.quantile(meds, [(1 - level) / 2, (1 + level) / 2])
    return float(np.median(x)), float(lo), float(hi)


@dataclass(frozen=True)
class Verdict:
    significant: bool
    cis_disjoint: bool
    above_floor: bool
    threshold_rel: float


def significance(a_ci: tuple[float, float], b_ci: tuple[float, float], rel_diff: float,
                 noise_floor_rel: float, factor: float) -> Verdict:
    disjoint = a_ci[1] < b_ci[0] or b_ci[1] < a_ci[0]
    threshold = factor * noise_floor_rel
    above = abs(rel_diff) > threshold
    return Verdict(disjoint and above, disjoint, above, threshold)


def time_launches(launch, outputs: list[Any], n_sets: int, params: MeasureParams = V1,
                  seed: int = 0, device: Any = None) -> dict[str, Any]:
    """The timing loop of src/kta/measure/bench.py:124-192 around ``launch(k)`` (the k-th
    launch, which picks input set k % n_sets itself): before every launch the ``outputs``
    (device tensors) are refilled with NaN bytes and a flush buffer of l2_flush_factor x L2
    bytes is written, then the single launch is timed between two CUDA events on the current
    stream; warm-up max(warmup_min_iters, warmup_min_ms), measured max(min_iters, min_ms);
    median with a bootstrap CI."""
    import torch

    from kta_b200 import runners

    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush_bytes = int(params.l2_flush_factor * l2)
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device=dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times: list[float] = []
    state = {"k": 0}

    def one(keep: bool) -> None:
        k = state["k"]
        state["k"] += 1
        if params.nan_fill:
            for b in outputs:
                b.view(torch.uint8).fill_(runners.NAN_BYTE)
        flush.fill_(k & 0xFF)
        start.record()
        launch(k)
        end.record()
        end.synchronize()
        if keep:
            times.append(start.elapsed_time(end))

    def phase(min_iters: int, min_ms: float, keep: bool) -> tuple[int, float]:
        n, t0 = 0, time.perf_counter()
        while n < params.max_iters and (n < min_iters or (time.perf_counter() - t0) * 1e3 < min_ms):
            one(keep)
            n += 1
        return n, time.perf_counter() - t0

    warm, warm_s = phase(params.warmup_min_iters, params.warmup_min_ms, False)
    iters, loop_s = phase(params.min_iters, params.min_ms, True)
    del flush
    times_us = [ms * 1e3 for ms in times]
    med, lo, hi = bootstrap_median(times_us, params.bootstrap_resamples, params.ci_level,
                                   random.Random(seed))
    return {"median_us": med, "ci_low_us": lo, "ci_high_us": hi, "n": len(times_us),
            "warmup_iters": warm, "warmup_s": warm_s, "loop_s": loop_s,
            "flush_bytes": flush_bytes, "input_sets": n_sets, "times_us": times_us}


def time_case(entry: str, problem, shape: dict[str, Any], sets: list[dict[str, np.ndarray]],
              params: MeasureParams = V1, seed: int = 0) -> dict[str, Any]:
    """Times ``entry`` under ``params`` on the host input sets ``sets`` (on cuda:0): the sets
    are copied to the device once, then ``time_launches`` rotates through them."""
    import torch

    from kta_b200 import inputs as kinp
    from kta_b200 import runners
    from kta_b200.reference import to_torch

    if len(sets) < params.min_input_sets:
        raise ValueError(f"the protocol wants >= {params.min_input_sets} input sets, "
                         f"got {len(sets)}")
    dev = torch.device("cuda")
    if "seqlens" in sets[0] and "max_seqlen" not in shape:
        shape = {**shape, "max_seqlen": int(max(np.max(s["seqlens"], initial=0) for s in sets))}
    dtypes = {t.name: t.dtype for t in problem.inputs}
    dsets = [{n: to_torch(a, dtypes[n], dev) for n, a in s.items()} for s in sets]
    outs = {}
    for t in problem.outputs:
        outs[t.name] = torch.empty(kinp.dims(t, shape), dtype=runners._TORCH[t.dtype], device=dev)
    fn = runners.resolve(entry)
    return time_launches(lambda k: fn(dsets[k % len(dsets)], shape, outs), list(outs.values()),
                         len(dsets), params, seed, dev)
