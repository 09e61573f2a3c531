"""Throughput of the libkta_b200 hot path on 1..8 B200 GPUs (one process per GPU).

Default workload: the bf16 GEMM case C = A . B^T at M = N = K = 8192 (kta_b200/cases/
gemm_bf16_8192.yaml), sharded across ranks by N-column blocks of B (rank r owns rows
[r N/n, (r+1) N/n) of B and the matching columns of C; A is replicated). No collective runs
on the data path; the total work is fixed as N grows ("scaling": "strong").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kta|reference]
                    [--workload gemm_bf16_8192|gemm_bf16_skinny|gemm_f16_1024|attn_causal|
                                decode_gqa|gemm_fp8|moe_gemm_f16|rmsnorm_f16|softmax_f16|
                                w4gemm_f16|nvfp4gemm_f16]

A step is one launch of the hot-path kernel over one rotating input set already resident in
HBM (at least 4 sets, and as many as make the sets together twice the 126 MB L2, so no flush
is needed between steps). Rank 0 prints one JSON line: the driver's keys plus `roofline` (the
dominant kernel's achieved rate from CUDA events against MEASURED_PEAKS.json), `sol` (the
case's L1 speed-of-light bound, as KTA reports pct_of_bound), `e2e` (the same metric through
the public API with pinned host inputs copied in and the result copied out every step, two
steps in flight on two streams), `cpu_baseline` (the reference's CPU torch path timed on a
bounded sample) and `clocks`.

`--impl reference` times the reference's own CPU implementation of the path instead: the
case statement run by torch on the host cores in the inputs' dtype, i.e. the "library"
statement of src/kta/checks/scripts/ref_torch.py:39-43 with the device set to cpu, each
step a bounded sample of the workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GEMM/attention TFLOP/s (decode: HBM GB/s) & % of SOL at 1/2/4/8 B200"
NSETS = int(os.environ.get("KTA_BENCH_SETS", "4"))  # rotating input sets (1 for ncu captures)
L2_BYTES = 126 * 1000 * 1000


def sets_for(bytes_per_set: float) -> int:
    """Rotating input sets: NSETS, raised until the sets together are twice the L2, so a step
    never finds its inputs left in L2 by the previous steps; KTA_BENCH_SETS set explicitly (a
    small ncu capture) wins."""
    if "KTA_BENCH_SETS" in os.environ:
        return NSETS
    return max(NSETS, int(-(-2 * L2_BYTES // max(int(bytes_per_set), 1))))


CPU_BUDGET_S = 12.0  # CPU baseline sample: about this much host compute
# Back-to-back launches before every timed region: the SM clock under the 1 kW power cap
# settles within about a second of sustained load; timing earlier catches a transient.
PREHEAT_S = 2.0


# ---------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------
class Dist:
    """One process per GPU: rank / world from torchrun's environment, a process group over
    NCCL (gloo when no GPU is present: the host-side logic is tested that way), max and sum
    reductions of per-rank scalars outside the timed region."""

    def __init__(self, want: int, backend: str | None = None) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if want > 1 and self.world != want:
            raise SystemExit(f"--gpus {want} needs torchrun with {want} ranks (WORLD_SIZE="
                             f"{self.world})")
        self.backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        self.pg = None

    def init(self) -> None:
        if self.world > 1:
            import datetime

            kw = {}
            if self.backend == "nccl":
                kw["device_id"] = torch.device("cuda", self.local)
            torch.distributed.init_process_group(
                self.backend, timeout=datetime.timedelta(seconds=120), **kw)
            self.pg = True

    def _dev(self) -> str:
        return "cuda" if self.backend == "nccl" else "cpu"

    def barrier(self) -> None:
        if self.pg:
            if self.backend == "nccl":
                torch.distributed.barrier(device_ids=[self.local])
            else:
                torch.distributed.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self._dev())
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self._dev())
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
        return float(t.item())

    def close(self) -> None:
        if self.pg:
            torch.distributed.destroy_process_group()


def shard(n: int, parts: int, i: int, align: int = 1) -> tuple[int, int]:
    """[lo, hi) of part i when n is split into `parts` blocks aligned to `align`."""
    units = -(-n // align)
    lo = (units * i) // parts * align
    hi = min(n, (units * (i + 1)) // parts * align)
    return lo, hi


# ---------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------
class Clocks:
    """SM clock, power and clock-event reasons of this rank's GPU, polled every 5 ms through
    NVML (read-only queries) on a background thread, so that even a timed region of a few
    milliseconds holds samples; nvidia-smi at its 100 ms floor is the fallback when NVML
    cannot be opened. Nothing here changes a GPU setting."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}
    PERIOD_S = 0.005

    def __init__(self) -> None:
        self.samples: list[tuple[float, dict[str, str]]] = []
        self.proc: subprocess.Popen | None = None
        self.thread: threading.Thread | None = None
        self.stop_flag = threading.Event()
        self.source = "none"
        self.bus: tuple[int, int, int] | None = None
        try:
            p = torch.cuda.get_device_properties(torch.cuda.current_device())
            self.bus = (int(p.pci_domain_id), int(p.pci_bus_id), int(p.pci_device_id))
        except Exception:
            self.bus = None

    def _mine(self, s: dict[str, str]) -> bool:
        if self.bus is None:
            return True
        try:  # nvidia-smi prints domain:bus:device.function in hex
            dom, bus, devfn = s["pci.bus_id"].split(":")
            return (int(dom, 16), int(bus, 16), int(devfn.split(".")[0], 16)) == self.bus
        except (KeyError, ValueError):
            return False

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        if self.bus is None:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(0)
        dom, bus, dev = self.bus
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0")

    def start(self) -> None:
        try:
            nv, h = self._nvml_handle()
            max_sm = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            bus_id = nv.nvmlDeviceGetPciInfo(h).busId
            bus_id = bus_id.decode() if isinstance(bus_id, bytes) else str(bus_id)
        except Exception:
            self._start_smi()
            return
        self.source = "nvml (5 ms)"

        def poll() -> None:
            while not self.stop_flag.is_set():
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = int(reasons_fn(h))
                except Exception:
                    break
                s = {"pci.bus_id": bus_id, "clocks.sm": str(sm), "clocks.max.sm": str(max_sm),
                     "power.draw": f"{pw:.2f}"}
                for k, bit in self.REASON_BITS.items():
                    s[f"clocks_event_reasons.{k}"] = "Active" if rs & bit else "Not Active"
                self.samples.append((time.time(), s))
                time.sleep(self.PERIOD_S)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()

    def _start_smi(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.source = "nvidia-smi (100 ms)"
        keys = self.FIELDS.split(",")

        def reader() -> None:
            assert self.proc is not None and self.proc.stdout is not None
            for line in self.proc.stdout:
                vals = [v.strip() for v in line.split(",")]
                if len(vals) == len(keys):
                    self.samples.append((time.time(), dict(zip(keys, vals))))

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self) -> None:
        self.stop_flag.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self, t0: float, t1: float) -> dict:
        mine = [s for t, s in self.samples if self._mine(s)]
        inside = [s for t, s in self.samples if t0 <= t <= t1 and self._mine(s)]
        use = inside or [s for t, s in self.samples if t0 - 0.15 <= t <= t1 + 0.15
                         and self._mine(s)] or mine[-3:]
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": self.source}

        def num(s: dict, k: str) -> float | None:
            try:
                return float(s[k])
            except (ValueError, KeyError):
                return None

        sm = [v for v in (num(s, "clocks.sm") for s in use) if v is not None]
        reasons = set()
        for s in use:
            for k in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                      "sw_power_cap", "hw_power_brake_slowdown"):
                if s.get(f"clocks_event_reasons.{k}", "").strip().lower() == "active":
                    reasons.add(k)
        power = [v for v in (num(s, "power.draw") for s in use) if v is not None]
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_mhz_min": min(sm) if sm else None,
            "sm_mhz_max": max(sm) if sm else None,
            "sm_max_mhz": num(use[0], "clocks.max.sm"),
            "reasons": sorted(reasons),
            "power_w_max": max(power) if power else None,
            "samples": len(use),
            "samples_in_timed_region": len(inside),
            "source": self.source,
        }


# ---------------------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------------------
def _randn(shape, dtype, gen, scale=1.0, device="cuda"):
    x = torch.randn(*shape, generator=gen, device=device, dtype=torch.float32)
    if scale != 1.0:
        x.mul_(scale)
    return x.to(dtype)


class GemmWorkload:
    """C = A . B^T (bf16/f16), this rank's N-column shard of B."""

    kernel_regex = "gemm"

    def __init__(self, name: str, m: int, n: int, k: int, dtype: torch.dtype, dist: Dist,
                 case: str) -> None:
        self.name, self.m, self.n_total, self.k, self.dtype = name, m, n, k, dtype
        self.case = case
        lo, hi = shard(n, dist.world, dist.rank, align=128)
        self.n0, self.n = lo, hi - lo
        self.esize = 2
        self.hbm_bound = m <= 64
        self.unit = "GB/s" if self.hbm_bound else "TFLOP/s"
        self.dtype_name = "bf16" if dtype == torch.bfloat16 else "f16"
        # a 1024^3 GEMM runs for a few microseconds: shorter than the host's launch path
        self.graph_default = 2.0 * m * n * k < 2e10
        self.nsets = sets_for((m * k + self.n * k + m * self.n) * self.esize)

    @property
    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    @property
    def bytes(self) -> float:
        return float((self.m * self.k + self.n * self.k + self.m * self.n) * self.esize)

    def work(self) -> float:  # this rank's units of the metric per step
        return self.bytes if self.hbm_bound else self.flops

    def sol_shape(self) -> dict:
        return {"M": self.m, "N": self.n, "K": self.k}

    def config(self, world: int) -> dict:
        return {
            "workload": f"{self.name}: C = A . B^T, {self.dtype_name}, M={self.m} N={self.n_total} "
                        f"K={self.k}, fp32 accumulate",
            "case": self.case,
            "M": self.m, "N": self.n_total, "K": self.k,
            "global_batch": self.m, "seq_len": None,
            "parallelism": f"N-column shards x{world} (no collective)",
            "l2": f"inputs larger than L2 (126 MB): {self.nsets} rotating input sets, no flush",
            "inputs": "N(0,1)/sqrt(K) from a seeded torch generator",
        }

    def setup(self, device: torch.device) -> None:
        g = torch.Generator(device=device).manual_seed(0)
        s = 1.0 / math.sqrt(self.k)
        self.a = [_randn((self.m, self.k), self.dtype, g, s) for _ in range(self.nsets)]
        self.b = [_randn((self.n, self.k), self.dtype, g, s) for _ in range(self.nsets)]
        self.c = [torch.empty((self.m, self.n), dtype=self.dtype, device=device)
                  for _ in range(self.nsets)]

    def launch(self, i: int) -> None:
        from kta_b200 import ops

        j = i % self.nsets
        ops.gemm(self.a[j], self.b[j], out=self.c[j])

    def gather_tensors(self) -> list[torch.Tensor]:
        """This rank's output block for the optional all-gather: C[:, n0:n0+n] of set 0."""
        return [self.c[0]]

    # ---- end to end: pinned host inputs in, result out, every step ----
    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        g = torch.Generator().manual_seed(seed)
        s = 1.0 / math.sqrt(self.k)
        self.ha = _randn((self.m, self.k), self.dtype, g, s, device="cpu").pin_memory()
        self.hb = _randn((self.n, self.k), self.dtype, g, s, device="cpu").pin_memory()
        self.hc = torch.empty((self.m, self.n), dtype=self.dtype).pin_memory()
        self.h2d_bytes = self.ha.numel() * self.esize + self.hb.numel() * self.esize
        self.d2h_bytes = self.hc.numel() * self.esize

    def e2e_step(self) -> None:
        from kta_b200 import ops

        # the public host-buffer entry: B, then A in row blocks copied in, each block's GEMM
        # as soon as it landed, C blocks copied out behind it (copies overlap compute); device
        # buffers of its own per caller stream; returns once queued, C valid on the host when
        # the caller's stream reaches this point
        ops.gemm_host(self.ha, self.hb, out=self.hc, wait=False)

    # ---- the reference's CPU torch path on a bounded sample ----
    def cpu_sample(self, rows: int):
        g = torch.Generator().manual_seed(7)
        s = 1.0 / math.sqrt(self.k)
        a = _randn((rows, self.k), self.dtype, g, s, device="cpu")
        b = _randn((self.n_total, self.k), self.dtype, g, s, device="cpu")

        def run():
            from oracle import statement

            statement.run_library("C = A @ B.T", {"A": a, "B": b}, {})

        units = (2.0 * rows * self.n_total * self.k if not self.hbm_bound
                 else float((rows * self.k + self.n_total * self.k + rows * self.n_total) * 2))
        return run, units, f"C = A @ B.T in {self.dtype_name} on the host, M={rows} rows of " \
                           f"A (of {self.m}), N={self.n_total}, K={self.k}"


def lpt(weights: list[int], parts: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of items to `parts` bins."""
    bins: list[list[int]] = [[] for _ in range(parts)]
    load = [0] * parts
    for i in sorted(range(len(weights)), key=lambda j: -weights[j]):
        t = min(range(parts), key=lambda r: load[r])
        bins[t].append(i)
        load[t] += weights[i]
    return [sorted(b) for b in bins]


class DecodeWorkload:
    """GQA decode: B=64, Hq=32, Hkv=8, D=128, lengths uniform in [1024, 8192] (seed 0);
    this rank's sequences by LPT on length."""

    kernel_regex = "decode_kernel"
    unit = "GB/s"
    dtype_name = "bf16"
    case = "decode_gqa"
    graph_default = False

    def __init__(self, dist: Dist, batch: int = 64, hq: int = 32, hkv: int = 8, d: int = 128,
                 lo: int = 1024, hi: int = 8192) -> None:
        import numpy as np

        self.batch, self.hq, self.hkv, self.d, self.max_seqlen = batch, hq, hkv, d, hi
        lengths = np.random.default_rng(0).integers(lo, hi + 1, size=batch)
        self.all_lengths = [int(x) for x in lengths]
        mine = lpt(self.all_lengths, dist.world)[dist.rank]
        self.lengths = [self.all_lengths[i] for i in mine]
        self.b = len(self.lengths)
        self.tokens = sum(self.lengths)

    @property
    def bytes(self) -> float:
        return float(2 * self.tokens * self.hkv * self.d * 2 + 2 * self.b * self.hq * self.d * 2
                     + self.b * 12)

    flops = None

    def work(self) -> float:
        return self.bytes

    def sol_shape(self) -> dict:
        return {"B": self.b, "Hq": self.hq, "Hkv": self.hkv, "D": self.d, "T": self.tokens,
                "max_seqlen": self.max_seqlen}

    def config(self, world: int) -> dict:
        return {"workload": f"decode_gqa: B={self.batch} Hq={self.hq} Hkv={self.hkv} D={self.d}, "
                            f"one query token, KV lengths U[1024, 8192] (seed 0), bf16 cache",
                "case": self.case, "B": self.batch, "Hq": self.hq, "Hkv": self.hkv, "D": self.d,
                "kv_tokens": sum(self.all_lengths), "global_batch": self.batch, "seq_len": None,
                "parallelism": f"sequences by LPT on length x{world} (no collective)",
                "l2": "inputs larger than L2: 4 rotating KV caches, no flush",
                "inputs": "N(0,1) bf16 from a seeded torch generator"}

    def _offsets(self):
        import numpy as np

        return np.concatenate([[0], np.cumsum(self.lengths)[:-1]]).astype(np.int64)

    def setup(self, device: torch.device) -> None:
        from kta_b200 import ops

        g = torch.Generator(device=device).manual_seed(0)
        self.q = [_randn((self.b, self.hq, self.d), torch.bfloat16, g) for _ in range(NSETS)]
        self.kc = [_randn((self.tokens, self.hkv, self.d), torch.bfloat16, g) for _ in range(NSETS)]
        self.vc = [_randn((self.tokens, self.hkv, self.d), torch.bfloat16, g) for _ in range(NSETS)]
        self.sl = torch.tensor(self.lengths, dtype=torch.int32, device=device)
        self.off = torch.tensor(self._offsets(), dtype=torch.int64, device=device)
        self.o = [torch.empty_like(self.q[0]) for _ in range(NSETS)]
        nbytes = ops.decode_workspace_bytes(self.b, self.hq, self.hkv, self.d, self.max_seqlen)
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)

    def launch(self, i: int) -> None:
        from kta_b200 import ops

        j = i % NSETS
        ops.decode_gqa(self.q[j], self.kc[j], self.vc[j], self.sl, self.off, self.max_seqlen,
                       out=self.o[j], workspace=self.ws)

    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        g = torch.Generator().manual_seed(seed)
        self.hq_ = _randn((self.b, self.hq, self.d), torch.bfloat16, g, device="cpu").pin_memory()
        self.hk = _randn((self.tokens, self.hkv, self.d), torch.bfloat16, g,
                         device="cpu").pin_memory()
        self.hv = _randn((self.tokens, self.hkv, self.d), torch.bfloat16, g,
                         device="cpu").pin_memory()
        # its own split-KV workspace: two end-to-end pipelines run at once and never share one
        from kta_b200 import ops

        self.ws = torch.zeros(ops.decode_workspace_bytes(self.b, self.hq, self.hkv, self.d,
                                                         self.max_seqlen),
                              dtype=torch.uint8, device=device)
        self.hsl = torch.tensor(self.lengths, dtype=torch.int32).pin_memory()
        self.hoff = torch.tensor(self._offsets(), dtype=torch.int64).pin_memory()
        self.ho = torch.empty((self.b, self.hq, self.d), dtype=torch.bfloat16).pin_memory()
        self.dq, self.dk, self.dv = (torch.empty_like(t, device=device)
                                     for t in (self.hq_, self.hk, self.hv))
        self.dsl = torch.empty_like(self.hsl, device=device)
        self.doff = torch.empty_like(self.hoff, device=device)
        self.do = torch.empty_like(self.ho, device=device)
        self.h2d_bytes = sum(t.numel() * t.element_size()
                             for t in (self.hq_, self.hk, self.hv, self.hsl, self.hoff))
        self.d2h_bytes = self.ho.numel() * 2

    def e2e_step(self) -> None:
        from kta_b200 import ops

        for dst, src in ((self.dq, self.hq_), (self.dk, self.hk), (self.dv, self.hv),
                         (self.dsl, self.hsl), (self.doff, self.hoff)):
            dst.copy_(src, non_blocking=True)
        ops.decode_gqa(self.dq, self.dk, self.dv, self.dsl, self.doff, self.max_seqlen,
                       out=self.do, workspace=self.ws)
        self.ho.copy_(self.do, non_blocking=True)

    def cpu_sample(self, nseq: int):
        """The decode case statement in bf16 on the host for the first `nseq` sequences."""
        nseq = max(1, min(nseq, self.b))
        lens = self.lengths[:nseq]
        g = torch.Generator().manual_seed(7)
        tot = sum(lens)
        q = _randn((nseq, self.hq, self.d), torch.bfloat16, g, device="cpu")
        kc = _randn((tot, self.hkv, self.d), torch.bfloat16, g, device="cpu")
        vc = _randn((tot, self.hkv, self.d), torch.bfloat16, g, device="cpu")
        import numpy as np

        off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        inputs = {"Q": q, "Kc": kc, "Vc": vc, "seqlens": torch.tensor(lens, dtype=torch.int32),
                  "kv_offsets": torch.tensor(off)}
        shape = {"B": nseq, "Hq": self.hq, "Hkv": self.hkv, "D": self.d}

        def run():
            from kta_b200 import schemas
            from oracle import statement

            stmt = schemas.load_case_file("decode_gqa").problem.reference_impl
            statement.run_library(stmt, inputs, shape, ["O"])

        units = float(2 * tot * self.hkv * self.d * 2 + 2 * nseq * self.hq * self.d * 2)
        return run, units, (f"decode statement in bf16 on the host for {nseq} of {self.b} "
                            f"sequences ({tot} KV tokens)")

    @property
    def m(self) -> int:  # the CPU calibration grows the sample up to all sequences
        return self.b


class AttnWorkload:
    """Causal attention forward, B=8 H=32 S=4096 D=128 bf16; this rank's batch x head
    slice (the heads are independent)."""

    kernel_regex = "attn_fwd_kernel"
    unit = "TFLOP/s"
    dtype_name = "bf16"
    case = "attn_causal"
    graph_default = False

    def __init__(self, dist: Dist, b: int = 8, h: int = 32, s: int = 4096, d: int = 128) -> None:
        self.b_total, self.h, self.s, self.d = b, h, s, d
        pairs = b * h
        lo, hi = shard(pairs, dist.world, dist.rank)
        # (batch, head) pairs lo .. hi - 1 in batch-major order; whole batches when the split
        # allows it (every N of 1, 2, 4, 8), otherwise heads of one batch entry
        self.pair_lo, self.pair_hi = lo, hi
        self.pairs = hi - lo
        if self.pairs % h == 0:
            self.b, self.hh = self.pairs // h, h
        else:
            self.b, self.hh = 1, self.pairs

    @property
    def flops(self) -> float:
        return 4.0 * self.b * self.hh * self.d * self.s * (self.s + 1) / 2

    @property
    def bytes(self) -> float:
        return float(4 * self.b * self.s * self.hh * self.d * 2 + self.b * self.hh * self.s * 4)

    def work(self) -> float:
        return self.flops

    def sol_shape(self) -> dict:
        return {"B": self.b, "S": self.s, "H": self.hh, "D": self.d}

    @property
    def m(self) -> int:
        return self.b * self.hh

    def config(self, world: int) -> dict:
        return {"workload": f"attn_causal: B={self.b_total} H={self.h} S={self.s} D={self.d}, "
                            "bf16, causal, O bf16 + LSE fp32",
                "case": self.case, "B": self.b_total, "H": self.h, "S": self.s, "D": self.d,
                "global_batch": self.b_total, "seq_len": self.s,
                "parallelism": f"batch x head shards x{world} (no collective)",
                "l2": "inputs larger than L2: 4 rotating Q/K/V sets (1.07 GB each), no flush",
                "inputs": "N(0,1) bf16 from a seeded torch generator"}

    def setup(self, device: torch.device) -> None:
        g = torch.Generator(device=device).manual_seed(0)
        shp = (self.b, self.s, self.hh, self.d)
        self.qkv = [[_randn(shp, torch.bfloat16, g) for _ in range(3)] for _ in range(NSETS)]
        self.o = [torch.empty(shp, dtype=torch.bfloat16, device=device) for _ in range(NSETS)]
        self.lse = [torch.empty((self.b, self.hh, self.s), dtype=torch.float32, device=device)
                    for _ in range(NSETS)]

    def launch(self, i: int) -> None:
        from kta_b200 import ops

        j = i % NSETS
        q, k, v = self.qkv[j]
        ops.attn_fwd_causal(q, k, v, out=self.o[j], lse=self.lse[j])

    def gather_tensors(self) -> list[torch.Tensor]:
        """This rank's O and LSE of set 0 (whole batch entries) for the optional all-gather."""
        return [self.o[0], self.lse[0]]

    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        g = torch.Generator().manual_seed(seed)
        shp = (self.b, self.s, self.hh, self.d)
        self.hqkv = [_randn(shp, torch.bfloat16, g, device="cpu").pin_memory() for _ in range(3)]
        self.ho = torch.empty(shp, dtype=torch.bfloat16).pin_memory()
        self.hl = torch.empty((self.b, self.hh, self.s), dtype=torch.float32).pin_memory()
        self.dqkv = [torch.empty_like(t, device=device) for t in self.hqkv]
        self.do = torch.empty_like(self.ho, device=device)
        self.dl = torch.empty_like(self.hl, device=device)
        self.h2d_bytes = 3 * self.hqkv[0].numel() * 2
        self.d2h_bytes = self.ho.numel() * 2 + self.hl.numel() * 4

    def e2e_step(self) -> None:
        from kta_b200 import ops

        for d, h in zip(self.dqkv, self.hqkv):
            d.copy_(h, non_blocking=True)
        ops.attn_fwd_causal(*self.dqkv, out=self.do, lse=self.dl)
        self.ho.copy_(self.do, non_blocking=True)
        self.hl.copy_(self.dl, non_blocking=True)

    def cpu_sample(self, pairs: int):
        """The case statement in bf16 on the host for `pairs` (batch, head) pairs."""
        pairs = max(1, min(pairs, self.b * self.hh))
        g = torch.Generator().manual_seed(7)
        shp = (1, self.s, pairs, self.d)
        q, k, v = (_randn(shp, torch.bfloat16, g, device="cpu") for _ in range(3))

        def run():
            from kta_b200 import schemas
            from oracle import statement

            stmt = schemas.load_case_file("attn_causal").problem.reference_impl
            statement.run_library(stmt, {"Q": q, "K": k, "V": v},
                                  {"B": 1, "S": self.s, "H": pairs, "D": self.d}, ["O", "LSE"])

        units = 4.0 * pairs * self.d * self.s * (self.s + 1) / 2
        return run, units, (f"causal attention statement in bf16 on the host for {pairs} of "
                            f"{self.b * self.hh} (batch, head) pairs, S={self.s}")


class Fp8Workload:
    """FP8 e4m3 block-scaled GEMM M=4096 N=7168 K=7168 (bf16 out); this rank's N-column
    shard, aligned to the 128-wide weight-scale blocks."""

    kernel_regex = "fp8_gemm_kernel"
    unit = "TFLOP/s"
    dtype_name = "e4m3"
    case = "gemm_fp8_blockscaled"
    graph_default = False
    peak_key = "fp8"

    def kernels_per_step(self) -> int:
        """The main launch, plus the quarter launch when the tiles of a ragged last round are
        cut into quarters (the rule of kta_gemm_fp8_blockscaled)."""
        tiles = -(-self.m // 128) * -(-self.n // 256)
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        rem = tiles % sms if tiles > sms else 0
        return 2 if rem > 0 and rem * 4 <= sms and os.environ.get("KTA_FP8_SPLIT") != "0" else 1

    def __init__(self, dist: Dist, m: int = 4096, n: int = 7168, k: int = 7168) -> None:
        self.m, self.n_total, self.k = m, n, k
        lo, hi = shard(n, dist.world, dist.rank, align=128)
        self.n0, self.n = lo, hi - lo

    @property
    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    @property
    def bytes(self) -> float:
        kb = -(-self.k // 128)
        return float(self.m * self.k + self.n * self.k + self.m * self.n * 2
                     + 4 * (self.m * kb + -(-self.n // 128) * kb))

    def work(self) -> float:
        return self.flops

    def sol_shape(self) -> dict:
        return {"M": self.m, "N": self.n, "K": self.k}

    def config(self, world: int) -> dict:
        return {"workload": f"gemm_fp8_blockscaled: M={self.m} N={self.n_total} K={self.k}, "
                            "e4m3 with fp32 scales per 1x128 (A) and 128x128 (B), bf16 out",
                "case": self.case, "M": self.m, "N": self.n_total, "K": self.k,
                "global_batch": self.m, "seq_len": None,
                "parallelism": f"N-column shards x{world} (no collective)",
                "l2": "inputs larger than L2: 4 rotating input sets (~88 MB each)",
                "inputs": "N(0,1) with 1% outliers x20, quantised on the device"}

    def _quant(self, x: torch.Tensor, rows: int):
        m, k = x.shape
        xb = x.view(m // rows if rows > 1 else m, rows, k // 128, 128) if rows > 1 else \
            x.view(m, 1, k // 128, 128)
        amax = xb.abs().amax(dim=(1, 3)).clamp_min(1e-30)
        scale = (amax / 448.0).float()
        q = (xb / scale[:, None, :, None]).view(m, k).to(torch.float8_e4m3fn)
        return q, scale.contiguous()

    def setup(self, device: torch.device) -> None:
        g = torch.Generator(device=device).manual_seed(0)
        self.sets = []
        for _ in range(NSETS):
            a = torch.randn(self.m, self.k, generator=g, device=device)
            a = torch.where(torch.rand(a.shape, generator=g, device=device) < 0.01, a * 20, a)
            b = torch.randn(self.n, self.k, generator=g, device=device)
            b = torch.where(torch.rand(b.shape, generator=g, device=device) < 0.01, b * 20, b)
            qa, sa = self._quant(a, 1)
            qb, sb = self._quant(b, 128)
            del a, b
            self.sets.append((qa, sa, qb, sb))
        self.c = [torch.empty((self.m, self.n), dtype=torch.bfloat16, device=device)
                  for _ in range(NSETS)]

    def launch(self, i: int) -> None:
        from kta_b200 import ops

        j = i % NSETS
        ops.gemm_fp8_blockscaled(*self.sets[j], out=self.c[j])

    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        qa, sa, qb, sb = self.sets[seed % len(self.sets)]  # each pipeline its own input set
        self.h = [t.cpu().pin_memory() for t in (qa.view(torch.uint8), sa, qb.view(torch.uint8), sb)]
        self.dv = [torch.empty_like(t, device=device) for t in self.h]
        self.hc = torch.empty((self.m, self.n), dtype=torch.bfloat16).pin_memory()
        self.dc = torch.empty_like(self.hc, device=device)
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.h)
        self.d2h_bytes = self.hc.numel() * 2

    def e2e_step(self) -> None:
        from kta_b200 import ops

        for d, h in zip(self.dv, self.h):
            d.copy_(h, non_blocking=True)
        ops.gemm_fp8_blockscaled(self.dv[0].view(torch.float8_e4m3fn), self.dv[1],
                                 self.dv[2].view(torch.float8_e4m3fn), self.dv[3], out=self.dc)
        self.hc.copy_(self.dc, non_blocking=True)

    def cpu_sample(self, rows: int):
        """The case statement (dequantise, then multiply) in fp32 on the host for `rows` rows
        of A: the inputs' own precision there is fp32 scales and e4m3 codes widened."""
        rows = max(1, min(rows, self.m))
        g = torch.Generator().manual_seed(7)
        a = torch.randn(rows, self.k, generator=g).to(torch.float8_e4m3fn).float()
        b = torch.randn(self.n_total, self.k, generator=g).to(torch.float8_e4m3fn).float()
        kb = -(-self.k // 128)
        sa = torch.rand(rows, kb, generator=g) + 0.5
        sb = torch.rand(-(-self.n_total // 128), kb, generator=g) + 0.5

        def run():
            from kta_b200 import schemas
            from oracle import statement

            stmt = schemas.load_case_file("gemm_fp8_blockscaled").problem.reference_impl
            statement.run_library(stmt, {"A": a, "sa": sa, "B": b, "sb": sb},
                                  {"M": rows, "N": self.n_total, "K": self.k}, ["C"])

        units = 2.0 * rows * self.n_total * self.k
        return run, units, (f"dequantise-and-multiply statement in fp32 on the host, M={rows} "
                            f"rows (of {self.m}), N={self.n_total}, K={self.k}")


class MoeWorkload:
    """MoE expert GEMM (KTA's moe_gemm, perfmodel/testset/gen.py:332-356) at the test set's
    shape E=8 T=2048 N=1024 K=2048, f16: T / E tokens per expert, W [E, K, N]; this rank's
    expert shard (experts are independent)."""

    kernel_regex = "gemm"
    unit = "TFLOP/s"
    dtype_name = "f16"
    case = "moe_gemm_f16"
    graph_default = True  # a few microseconds per launch: shorter than the host launch path

    def __init__(self, dist: Dist, e: int = 8, t: int = 2048, n: int = 1024, k: int = 2048):
        self.e_total, self.t_total, self.n, self.k = e, t, n, k
        lo, hi = shard(e, dist.world, dist.rank)
        self.e = max(hi - lo, 0)
        self.t = self.e * (t // e)
        self.m = self.t
        self.nsets = sets_for((self.t * k + self.e * k * n + self.t * n) * 2)

    @property
    def flops(self) -> float:
        return 2.0 * self.t * self.n * self.k

    @property
    def bytes(self) -> float:
        return float((self.t * self.k + self.e * self.k * self.n + self.t * self.n) * 2)

    def work(self) -> float:
        return self.flops

    def sol_shape(self) -> dict:
        return {"E": self.e, "T": self.t, "N": self.n, "K": self.k}

    def config(self, world: int) -> dict:
        return {"workload": f"moe_gemm_f16: E={self.e_total} T={self.t_total} N={self.n} "
                            f"K={self.k}, f16, fp32 accumulate",
                "case": self.case, "E": self.e_total, "T": self.t_total, "N": self.n,
                "K": self.k, "global_batch": self.t_total, "seq_len": None,
                "parallelism": f"expert shards x{world} (no collective)",
                "l2": f"inputs larger than L2 together: {self.nsets} rotating input sets",
                "inputs": "N(0,1)/sqrt(K) f16 from a seeded torch generator"}

    def setup(self, device: torch.device) -> None:
        g = torch.Generator(device=device).manual_seed(0)
        s = 1.0 / math.sqrt(self.k)
        self.a = [_randn((self.t, self.k), torch.float16, g, s) for _ in range(self.nsets)]
        self.w = [_randn((self.e, self.k, self.n), torch.float16, g, s)
                  for _ in range(self.nsets)]
        self.c = [torch.empty((self.t, self.n), dtype=torch.float16, device=device)
                  for _ in range(self.nsets)]

    def launch(self, i: int) -> None:
        from kta_b200 import ops

        j = i % self.nsets
        ops.moe_gemm(self.a[j], self.w[j], out=self.c[j])

    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        g = torch.Generator().manual_seed(seed)
        s = 1.0 / math.sqrt(self.k)
        self.ha = _randn((self.t, self.k), torch.float16, g, s, device="cpu").pin_memory()
        self.hw = _randn((self.e, self.k, self.n), torch.float16, g, s, device="cpu").pin_memory()
        self.hc = torch.empty((self.t, self.n), dtype=torch.float16).pin_memory()
        self.da = torch.empty_like(self.ha, device=device)
        self.dw = torch.empty_like(self.hw, device=device)
        self.dc = torch.empty_like(self.hc, device=device)
        self.h2d_bytes = (self.ha.numel() + self.hw.numel()) * 2
        self.d2h_bytes = self.hc.numel() * 2

    def e2e_step(self) -> None:
        from kta_b200 import ops

        self.da.copy_(self.ha, non_blocking=True)
        self.dw.copy_(self.hw, non_blocking=True)
        ops.moe_gemm(self.da, self.dw, out=self.dc)
        self.hc.copy_(self.dc, non_blocking=True)

    def cpu_sample(self, rows: int):
        g = torch.Generator().manual_seed(7)
        s = 1.0 / math.sqrt(self.k)
        per = self.t_total // self.e_total
        rows = max(1, min(rows, per))
        a = _randn((rows, self.k), torch.float16, g, s, device="cpu")
        w = _randn((self.k, self.n), torch.float16, g, s, device="cpu")

        def run():
            from oracle import statement

            statement.run_library("C = A @ W", {"A": a, "W": w}, {})

        units = 2.0 * rows * self.n * self.k
        return run, units, (f"one expert's A @ W[e] in f16 on the host, {rows} of its {per} "
                            f"rows, N={self.n}, K={self.k}")


class Dq4Workload:
    """GEMM with a 4-bit B dequantised in the main loop (KTA's test-set w4gemm, group 32, and
    nvfp4gemm, e2m1 with 16-element blocks; perfmodel/testset/gen.py:359-414, :744-778) at the
    test set's M=N=K=2048, f16 A, scales and C; this rank's N-column shard of B."""

    kernel_regex = "dq_gemm_kernel"
    unit = "TFLOP/s"
    dtype_name = "f16"
    graph_default = True  # ~20 us per launch: near the host launch path

    def __init__(self, fmt: str, dist: Dist, m: int = 2048, n: int = 2048,
                 k: int = 2048) -> None:
        self.fmt = fmt
        self.group = 32 if fmt == "int4" else 16
        self.case = "w4gemm_f16" if fmt == "int4" else "nvfp4gemm_f16"
        self.m, self.n_total, self.k = m, n, k
        lo, hi = shard(n, dist.world, dist.rank, align=128)
        self.n0, self.n = lo, hi - lo
        self.nsets = sets_for(2 * m * k + self.n * k // 2 + 2 * self.n * (k // self.group)
                              + 2 * m * self.n)

    @property
    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    @property
    def bytes(self) -> float:
        return float(2 * self.m * self.k + self.n * self.k // 2
                     + 2 * self.n * (self.k // self.group) + 2 * self.m * self.n)

    def work(self) -> float:
        return self.flops

    def sol_shape(self) -> dict:
        return {"M": self.m, "N": self.n, "K": self.k}

    def config(self, world: int) -> dict:
        what = ("w4a16: B = (nibble - 8) * scale per 32 along K" if self.fmt == "int4"
                else "NVFP4: B = e2m1(nibble) * scale per 16 along K")
        return {"workload": f"{self.case}: M={self.m} N={self.n_total} K={self.k}, {what}, "
                            "f16 A / scales / C, fp32 accumulate",
                "case": self.case, "M": self.m, "N": self.n_total, "K": self.k,
                "global_batch": self.m, "seq_len": None,
                "parallelism": f"N-column shards x{world} (no collective)",
                "l2": f"inputs larger than L2 together: {self.nsets} rotating input sets",
                "inputs": "A N(0,1)/sqrt(K) f16 (seeded torch); B N(0,1) quantised on the host"}

    def _quantised(self, n: int, seed: int):
        from kta_b200.inputs import quantize_4bit

        src = np.random.default_rng(seed).standard_normal((n, self.k)).astype(np.float32)
        bq, sc = quantize_4bit(src, self.fmt, self.group)
        return torch.from_numpy(bq), torch.from_numpy(sc)

    def setup(self, device: torch.device) -> None:
        g = torch.Generator(device=device).manual_seed(0)
        s = 1.0 / math.sqrt(self.k)
        hbq, hsc = self._quantised(self.n, 11)
        self.sets = [(_randn((self.m, self.k), torch.float16, g, s), hbq.to(device),
                      hsc.to(device)) for _ in range(self.nsets)]
        self.c = [torch.empty((self.m, self.n), dtype=torch.float16, device=device)
                  for _ in range(self.nsets)]

    def launch(self, i: int) -> None:
        from kta_b200 import ops

        j = i % self.nsets
        ops.gemm_4bit(*self.sets[j], self.fmt, self.group, out=self.c[j])

    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        g = torch.Generator().manual_seed(seed)
        self.ha = _randn((self.m, self.k), torch.float16, g, 1.0 / math.sqrt(self.k),
                         device="cpu").pin_memory()
        bq, sc = self._quantised(self.n, 12)
        self.hbq, self.hsc = bq.pin_memory(), sc.pin_memory()
        self.hc = torch.empty((self.m, self.n), dtype=torch.float16).pin_memory()
        self.da, self.dbq, self.dsc, self.dc = (torch.empty_like(t, device=device)
                                                for t in (self.ha, self.hbq, self.hsc, self.hc))
        self.h2d_bytes = self.ha.numel() * 2 + self.hbq.numel() + self.hsc.numel() * 2
        self.d2h_bytes = self.hc.numel() * 2

    def e2e_step(self) -> None:
        from kta_b200 import ops

        self.da.copy_(self.ha, non_blocking=True)
        self.dbq.copy_(self.hbq, non_blocking=True)
        self.dsc.copy_(self.hsc, non_blocking=True)
        ops.gemm_4bit(self.da, self.dbq, self.dsc, self.fmt, self.group, out=self.dc)
        self.hc.copy_(self.dc, non_blocking=True)

    def cpu_sample(self, rows: int):
        """The case statement (unpack, dequantise in f16, multiply) on the host for `rows`
        rows of A against the whole B."""
        rows = max(1, min(rows, self.m))
        g = torch.Generator().manual_seed(7)
        a = _randn((rows, self.k), torch.float16, g, 1.0 / math.sqrt(self.k), device="cpu")
        bq, sc = self._quantised(self.n_total, 13)

        def run():
            from kta_b200 import schemas
            from oracle import statement

            stmt = schemas.load_case_file(self.case).problem.reference_impl
            statement.run_library(stmt, {"A": a, "Bq": bq, "Sc": sc},
                                  {"M": rows, "N": self.n_total, "K": self.k}, ["C"])

        units = 2.0 * rows * self.n_total * self.k
        return run, units, (f"{self.case} statement in f16 on the host, M={rows} rows (of "
                            f"{self.m}), N={self.n_total}, K={self.k}")


class RowOpWorkload:
    """Row RMSNorm or softmax over X [M, N] f16 (KTA's test-set rmsnorm / softmax,
    perfmodel/testset/gen.py:662-704, :781-807) at an HBM-bound size; this rank's row shard.
    HBM-bound: X read once, Y written once (W once for RMSNorm)."""

    unit = "GB/s"
    dtype_name = "f16"
    graph_default = False
    hbm_bound = True

    def __init__(self, op: str, dist: Dist, m: int = 65536, n: int = 4096) -> None:
        self.op, self.m_total, self.n = op, m, n
        lo, hi = shard(m, dist.world, dist.rank)
        self.m = hi - lo
        self.case = f"{op}_f16"
        self.kernel_regex = "rowop_kernel"

    @property
    def flops(self) -> float:
        return 0.0

    @property
    def bytes(self) -> float:
        return float(2 * self.m * self.n * 2 + (self.n * 2 if self.op == "rmsnorm" else 0))

    def work(self) -> float:
        return self.bytes

    def sol_shape(self) -> dict:
        return {"M": self.m, "N": self.n}

    def config(self, world: int) -> dict:
        what = ("Y = X * rsqrt(mean(X^2) + 1e-6) * W" if self.op == "rmsnorm"
                else "Y = softmax(X) per row")
        return {"workload": f"{self.op}_f16: {what}, f16, M={self.m_total} N={self.n}, fp32 "
                            "statistics",
                "case": self.case, "M": self.m_total, "N": self.n,
                "global_batch": self.m_total, "seq_len": None,
                "parallelism": f"row shards x{world} (no collective)",
                "l2": "inputs larger than L2: 4 rotating X/Y sets (512 MB each), no flush",
                "inputs": "N(0,1) f16 from a seeded torch generator"}

    def setup(self, device: torch.device) -> None:
        g = torch.Generator(device=device).manual_seed(0)
        self.x = [_randn((self.m, self.n), torch.float16, g) for _ in range(NSETS)]
        self.y = [torch.empty((self.m, self.n), dtype=torch.float16, device=device)
                  for _ in range(NSETS)]
        self.w = _randn((self.n,), torch.float16, g)

    def _run(self, x, y) -> None:
        from kta_b200 import ops

        if self.op == "rmsnorm":
            ops.rmsnorm(x, self.w, 1e-6, out=y)
        else:
            ops.softmax(x, out=y)

    def launch(self, i: int) -> None:
        j = i % NSETS
        self._run(self.x[j], self.y[j])

    def setup_e2e(self, device: torch.device, seed: int = 99) -> None:
        g = torch.Generator().manual_seed(seed)
        self.hx = _randn((self.m, self.n), torch.float16, g, device="cpu").pin_memory()
        self.hy = torch.empty((self.m, self.n), dtype=torch.float16).pin_memory()
        self.dx = torch.empty_like(self.hx, device=device)
        self.dy = torch.empty_like(self.hy, device=device)
        self.h2d_bytes = self.hx.numel() * 2
        self.d2h_bytes = self.hy.numel() * 2

    def e2e_step(self) -> None:
        self.dx.copy_(self.hx, non_blocking=True)
        self._run(self.dx, self.dy)
        self.hy.copy_(self.dy, non_blocking=True)

    def cpu_sample(self, rows: int):
        rows = max(1, min(rows, self.m_total))
        g = torch.Generator().manual_seed(7)
        x = _randn((rows, self.n), torch.float16, g, device="cpu")
        w = _randn((self.n,), torch.float16, g, device="cpu")

        def run():
            from kta_b200 import schemas
            from oracle import statement

            stmt = schemas.load_case_file(self.case).problem.reference_impl
            tensors = {"X": x, "W": w} if self.op == "rmsnorm" else {"X": x}
            statement.run_library(stmt, tensors, {"M": rows, "N": self.n})

        units = float(2 * rows * self.n * 2)
        return run, units, (f"{self.op} statement in f16 on the host for {rows} of "
                            f"{self.m_total} rows, N={self.n}")


WORKLOADS = {
    "gemm_bf16_8192": lambda d: GemmWorkload("gemm_bf16_8192", 8192, 8192, 8192,
                                             torch.bfloat16, d, "gemm_bf16_8192"),
    "gemm_bf16_skinny": lambda d: GemmWorkload("gemm_bf16_skinny", 16, 8192, 8192,
                                               torch.bfloat16, d, "gemm_bf16_8192"),
    "gemm_f16_1024": lambda d: GemmWorkload("gemm_f16_1024", 1024, 1024, 1024,
                                            torch.float16, d, "gemm_f16_1024"),
    "decode_gqa": lambda d: DecodeWorkload(d),
    "attn_causal": lambda d: AttnWorkload(d),
    "gemm_fp8": lambda d: Fp8Workload(d),
    "moe_gemm_f16": lambda d: MoeWorkload(d),
    "rmsnorm_f16": lambda d: RowOpWorkload("rmsnorm", d),
    "softmax_f16": lambda d: RowOpWorkload("softmax", d),
    "w4gemm_f16": lambda d: Dq4Workload("int4", d),
    "nvfp4gemm_f16": lambda d: Dq4Workload("e2m1", d),
}


# ---------------------------------------------------------------------------------------
# measurement
# ---------------------------------------------------------------------------------------
def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 0) or 0),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback (profiling recipe: 6.65 TB/s, 1.59 PFLOP/s)"}


def traffic_for(workload: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    e = d.get(workload)
    return float(e["dram_bytes_per_launch"]) if e else None


def time_device(wl, steps: int, warmup: int, dist: Dist) -> dict:
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        wl.launch(i)
    # keep the GPU busy for PREHEAT_S more, back to back, so that the clock has settled under
    # the power cap before the timed launches (the sustained regime, not a transient)
    torch.cuda.synchronize()
    t_w = time.perf_counter()
    i = 0
    while time.perf_counter() - t_w < PREHEAT_S:
        wl.launch(i)
        i += 1
        if i % 8 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    wall0 = time.time()
    evs[0].record(stream)
    for s in range(steps):
        wl.launch(s)
        evs[s + 1].record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    dist.barrier()
    torch.cuda.synchronize()
    per = [evs[s].elapsed_time(evs[s + 1]) for s in range(steps)]
    total_ms = evs[0].elapsed_time(evs[steps])
    return {"total_ms": total_ms, "per_launch_ms": per, "wall": (wall0, wall1)}


def time_device_graph(wl, steps: int, warmup: int, dist: Dist) -> dict:
    """The K steps captured once into a CUDA graph and replayed: for launch-bound workloads
    whose kernels are shorter than the host's launch path."""
    for i in range(warmup):
        wl.launch(i)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for s in range(steps):
                wl.launch(s)
    torch.cuda.synchronize()
    graph.replay()  # warm replay
    t_w = time.perf_counter()
    while time.perf_counter() - t_w < PREHEAT_S:
        graph.replay()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    dist.barrier()
    total = e0.elapsed_time(e1)
    del graph
    return {"total_ms": total, "per_launch_ms": [total / steps] * steps, "wall": (wall0, wall1),
            "graph": True}


def time_e2e(wl, steps: int, dist: Dist, device: torch.device) -> dict:
    """Steps through the public API with pinned host buffers, each step copying its inputs
    in and its result out. Consecutive steps alternate between two pipelines (own host and
    device buffers, own stream), as a serving loop overlaps them: one step's read-back runs
    beside the next step's upload on the full-duplex link."""
    import copy

    main = torch.cuda.current_stream()
    pipes = [wl, copy.copy(wl)]
    # new buffers and different inputs on the copy; the workload keeps its own
    pipes[1].setup_e2e(device, seed=100)
    streams = [torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)]

    def run(n: int) -> None:
        for st in streams:
            st.wait_stream(main)
        for s in range(n):
            with torch.cuda.stream(streams[s % 2]):
                pipes[s % 2].e2e_step()
        for st in streams:
            main.wait_stream(st)

    run(2)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    run(steps)
    e1.record(main)
    torch.cuda.synchronize()
    dist.barrier()
    return {"total_ms": e0.elapsed_time(e1), "pipelines": 2}


def wl_kernels_per_step(wl) -> int:
    """Kernels of this library one step launches: 1, or the workload's own count."""
    fn = getattr(wl, "kernels_per_step", None)
    return int(fn()) if callable(fn) else 1


def gather_outputs(wl, dist: Dist, reps: int = 5) -> dict | None:
    """The optional all-gather of every rank's output block over NCCL (torch.distributed,
    NVLink), timed on its own after the timed region: `reps` all-gathers of the workload's
    gather_tensors() between CUDA events, max over ranks. Not part of `value`."""
    if dist.world == 1 or not dist.pg or not hasattr(wl, "gather_tensors"):
        return None
    local = wl.gather_tensors()
    bufs = [[torch.empty_like(t) for _ in range(dist.world)] for t in local]

    def once() -> None:
        for t, b in zip(local, bufs):
            torch.distributed.all_gather(b, t)

    once()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        once()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1) / reps)
    nbytes = sum(t.numel() * t.element_size() for t in local)
    # bitwise: output sets the protocol left NaN-filled must compare equal too
    ok = all(torch.equal(b[dist.rank].contiguous().view(torch.uint8), t.contiguous().view(torch.uint8))
             for t, b in zip(local, bufs))
    return {"ms": round(ms, 4), "bytes_per_rank": nbytes,
            "algbw_gbs": round(nbytes * dist.world / (ms * 1e6), 2),
            "busbw_gbs": round(nbytes * (dist.world - 1) / (ms * 1e6), 2),
            "own_block_intact": ok, "reps": reps,
            "what": "torch.distributed.all_gather (NCCL) of each rank's output block"}


def time_protocol(wl) -> dict:
    """The reference's measurement protocol (src/kta/measure/protocol.py:27-45, the timing loop
    of src/kta/measure/bench.py:124-192, kta_b200.measure.time_launches) on this workload's
    own rotating device sets: before every launch its outputs are NaN-filled and a 2 x L2
    flush buffer is written; each launch is timed alone between two CUDA events; warm-up
    >= 10 iterations and 50 ms, measured >= 100 iterations and 200 ms; median with a bootstrap
    95 % CI."""
    from kta_b200 import measure

    outs = [t for name in ("c", "o", "lse", "y") for t in (getattr(wl, name, None) or [])
            if isinstance(t, torch.Tensor)]
    nsets = getattr(wl, "nsets", NSETS)
    res = measure.time_launches(wl.launch, outs, nsets, measure.V1, seed=0)
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    return {
        "median_us": round(res["median_us"], 3),
        "ci_low_us": round(res["ci_low_us"], 3),
        "ci_high_us": round(res["ci_high_us"], 3),
        "value_at_median": round(wl.work() / (res["median_us"] * 1e-6) / scale, 3),
        "unit": wl.unit,
        "n": res["n"],
        "warmup_iters": res["warmup_iters"],
        "input_sets": nsets,
        "flush_bytes": res["flush_bytes"],
        "protocol": "KTA measure protocol: NaN-filled outputs and a 2 x L2 flush before "
                    "every launch, one launch between two CUDA events, warm-up >= 10 it and "
                    "50 ms, >= 100 it and 200 ms, median + bootstrap 95% CI (1000 resamples)",
    }


def calibrate_cpu(wl, budget_s: float):
    """A sample of the workload (rows of the first operand, then repeats of the whole
    workload) sized to about ``budget_s`` seconds of host compute."""
    full = getattr(wl, "m", 8)
    rows = min(8, full)
    run, units, sample = wl.cpu_sample(rows)
    run()  # first call pays library initialisation
    while True:
        t = time.perf_counter()
        run()
        dt = max(time.perf_counter() - t, 1e-6)
        if dt >= 0.25 or rows >= full:
            break
        rows = min(full, rows * 4)
        run, units, sample = wl.cpu_sample(rows)
    if rows < full:
        new_rows = min(full, max(8, int(rows * budget_s / dt) // 8 * 8))
        dt = dt * new_rows / rows
        rows = new_rows
        run, units, sample = wl.cpu_sample(rows)
    repeats = max(1, int(budget_s / dt)) if rows >= full else 1
    return run, units, sample, repeats


def cpu_baseline(wl, budget_s: float) -> dict:
    """The reference's CPU torch path timed on a bounded sample of ~budget_s seconds."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    run, units, sample, repeats = calibrate_cpu(wl, budget_s)
    t = time.perf_counter()
    for _ in range(repeats):
        run()
    dt = time.perf_counter() - t
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    return {"value": units * repeats / dt / scale, "unit": wl.unit,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{sample}; {repeats} repetition(s)", "seconds": round(dt, 3),
            "host_cpus": os.cpu_count()}


def run_kta(args, dist: Dist) -> dict | None:
    from kta_b200 import bound as kbound, lib, schemas

    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    dist.init()
    lib.load()
    wl = WORKLOADS[args.workload](dist)
    wl.setup(device)
    if args.profile:
        # exactly W + K launches of the hot-path kernel, nothing else (for ncu captures)
        for i in range(args.warmup + args.steps):
            wl.launch(i)
        torch.cuda.synchronize()
        print(json.dumps({"profile": args.workload, "launches": args.warmup + args.steps}))
        return None
    use_graph = args.graph or getattr(wl, "graph_default", False)
    clocks = Clocks()
    clocks.start()
    if use_graph:
        dev = time_device_graph(wl, args.steps, args.warmup, dist)
    else:
        dev = time_device(wl, args.steps, args.warmup, dist)
    clocks.stop()
    ms_total = dist.max(dev["total_ms"])
    world_work = dist.sum(wl.work())
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = world_work * args.steps / (ms_total / 1e3) / scale
    per = sorted(dev["per_launch_ms"])
    mean_launch_ms = sum(per) / len(per)
    pk = peaks()
    peak = pk["bf16_tflops"] if wl.unit == "TFLOP/s" else pk["hbm_gbs"]
    peak_note = "bf16_tflops (burst)" if wl.unit == "TFLOP/s" else "hbm_gbs"
    if getattr(wl, "peak_key", None) == "fp8":
        peak, peak_note = 2 * pk["bf16_tflops"], "2 x bf16_tflops (dense fp8 = 2x bf16 rate)"
    achieved = wl.work() / (mean_launch_ms / 1e3) / scale
    traffic = traffic_for(args.workload)
    roofline = {
        "kernel": wl.kernel_regex,
        "bound": "tensor" if wl.unit == "TFLOP/s" else "hbm",
        "achieved": round(achieved, 2),
        "peak": peak,
        "unit": wl.unit,
        "frac": round(achieved / peak, 4),
        "peak_source": f"{pk['source']}: {peak_note}",
        "traffic": traffic,
        "algorithmic_bytes_per_launch": wl.bytes,
        "algorithmic_flops_per_launch": getattr(wl, "flops", None),
        "mean_launch_ms": round(mean_launch_ms, 5),
        "timing": ("one CUDA graph of the K launches, total / K" if use_graph else
                   "CUDA events between consecutive launches on the launching stream")
                  + f", after {PREHEAT_S:.1f} s of back-to-back launches",
        "median_launch_ms": round(statistics.median(per), 5),
    }
    if wl.unit == "TFLOP/s" and pk["bf16_tflops_sustained"] > 0:
        # the timed launches run back to back under the power cap, as the sustained cuBLAS
        # figure was taken; `frac` stays against the burst figure
        sus = pk["bf16_tflops_sustained"] * (2 if getattr(wl, "peak_key", None) == "fp8" else 1)
        roofline["peak_sustained"] = sus
        roofline["frac_of_sustained"] = round(achieved / sus, 4)
    # the same K launches captured once as a CUDA graph and replayed back to back
    graph_b2b = None
    if not use_graph and not args.no_extra:
        g = time_device_graph(wl, args.steps, args.warmup, dist)
        g_ms = dist.max(g["total_ms"])
        graph_b2b = {"value": round(world_work * args.steps / (g_ms / 1e3) / scale, 3),
                     "unit": wl.unit, "ms_per_launch": round(g_ms / args.steps, 5),
                     "launches": args.steps}
    # the reference's own timing protocol on the same sets (this rank's figure)
    protocol = None if args.no_extra else time_protocol(wl)
    # the optional all-gather of the output blocks, timed on its own
    gathered = None if args.no_extra else gather_outputs(wl, dist)
    # KTA's L1 speed-of-light bound of this rank's shard, as pct_of_bound
    cf = schemas.load_case_file(wl.case)
    hw = kbound.b200_model()
    sol = kbound.sol_report(cf.problem, wl.sol_shape(), statistics.median(per) * 1e3, hw)
    # end to end through the public API with host buffers
    wl.setup_e2e(device)
    e2e_steps = max(3, min(args.steps, 20))
    e2e = time_e2e(wl, e2e_steps, dist, device)
    e2e_ms = dist.max(e2e["total_ms"])
    e2e_value = world_work * e2e_steps / (e2e_ms / 1e3) / scale
    result = None
    if dist.rank == 0:
        cpu = cpu_baseline(wl, CPU_BUDGET_S) if dist.world == 1 else None
        ck = clocks.summary(*dev["wall"])
        result = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": wl.unit,
            "n_gpus": dist.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_total / args.steps, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": wl.dtype_name,
            "data": "synthetic: the case's distributions from a torch generator seeded with 0",
            "config": wl.config(dist.world),
            "impl": "kta",
            "roofline": roofline,
            "sol": {"pct_of_bound": round(sol["pct_of_bound"], 2), "bound_us": sol["bound_us"],
                    "bottleneck": sol["bottleneck"], "near_bound": sol["near_bound"],
                    "per_rank_shape": wl.sol_shape(), "peak_sources": sol["peak_sources"]},
            "e2e": {"value": round(e2e_value, 3), "unit": wl.unit,
                    "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes,
                    "steps": e2e_steps,
                    "path": "pinned host -> device copies, libkta_b200 C-ABI launch, "
                            "device -> pinned host copy, every step; consecutive steps on "
                            "two streams with their own buffers (one step's read-back "
                            "beside the next one's upload)",
                    "pipelines": e2e.get("pipelines", 1)},
            "cpu_baseline": cpu,
            "clocks": ck,
            "gpu_launches": args.steps * wl_kernels_per_step(wl),
            "graph_b2b": graph_b2b,
            "protocol": protocol,
            "allgather": gathered,
        }
    return result


def run_reference(args, dist: Dist) -> dict | None:
    """The reference's CPU implementation of the path (the case statement in the inputs'
    dtype through torch on the host cores); rank 0 only."""
    if dist.rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    wl = WORKLOADS[args.workload](Dist(1))
    budget_per_step = max(0.05, 150.0 / max(1, args.steps + args.warmup))
    run, units, sample, repeats = calibrate_cpu(wl, budget_per_step)
    units *= repeats
    sample = f"{sample}; {repeats} repetition(s)"

    def step() -> None:
        for _ in range(repeats):
            run()

    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = units * args.steps / dt / scale
    return {
        "metric": METRIC,
        "value": round(value, 4),
        "unit": wl.unit,
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": wl.dtype_name,
        "data": "synthetic: the case's distributions from a torch generator seeded with 0",
        "config": wl.config(1),
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": wl.unit, "cores": threads,
                         "kind": "port", "sample": f"per step: {sample}"},
        "e2e": {"value": round(value, 4), "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["kta", "reference"], default="kta")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="gemm_bf16_8192")
    ap.add_argument("--graph", action="store_true",
                    help="time the K steps as one CUDA graph replay (launch-bound workloads)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the CUDA-graph back-to-back figure and the protocol median")
    ap.add_argument("--profile", action="store_true",
                    help="run W + K launches of the kernel only (the command for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    dist = Dist(args.gpus)
    if args.impl == "reference":
        out = run_reference(args, dist)
    else:
        out = run_kta(args, dist)
    if out is not None:
        print(json.dumps(out), flush=True)
    if args.impl == "kta":
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
