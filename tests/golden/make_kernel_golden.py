"""Fixtures from the reference's own kernels: runs KTA's TileLang test-set kernels on a GPU and
records their inputs and outputs, to pin the oracle's attention, decode and FP8 restatements.

    python tests/golden/make_kernel_golden.py <path of KTA's perfmodel/testset/gen.py> <out.npz>

Needs a CUDA GPU and TileLang (the reference pins 0.1.15; this image has 0.1.9, which lowers
these kernels for sm_100a with the reference's own pass configs, gen.py:PASS_CONFIGS: no TMA
lowering, no warp specialisation). The script only calls gen.py's kernel builders and
`tilelang.compile(func, target="cuda", pass_configs=PASS_CONFIGS)` as gen.py's `_compiled`
does (gen.py:915-918); nothing of gen.py is copied. Kernels and shapes:

- ``fa_forward`` (gen.py:417-486): B=1, S=256, H=2, D=128, BM=BN=64, 2 stages, 128 threads
  (the test set's FA tile, gen.py FA); fp16 Q, K, V ~ N(0, 1); non-causal; Out fp16.
- ``decode_partial`` + ``decode_combine`` (gen.py:493-590): B=1, H=8 query heads, G=2 KV
  heads, S=512, D=128, BN=BH=64, split=4, 2 stages (the test set's DECODE tile); fp16 Q, K, V
  ~ N(0, 1); glse (log2 units, fp16), Opart (fp16), Out (fp16). Q sits at the start of a
  larger zeroed allocation: the kernel's Q tile is BH rows starting at a head of the batch
  entry, more rows than the entry has.
- ``fp8gemm`` (gen.py:306-329) at M = N = K = 256 (gen.py's SHAPE set for this run), tile
  128x128x64, 3 stages, 128 threads: A [M, K], B [N, K] e4m3 codes of N(0, 1) draws, C fp16.

The inputs come from numpy generators seeded per kernel and are stored as raw bits next to
the outputs.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np


def _load_gen(path: str):
    spec = importlib.util.spec_from_file_location("kta_testset_gen", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _compile(g, func):
    import tilelang

    return tilelang.compile(func, target="cuda", pass_configs=g.PASS_CONFIGS)


def main(gen_path: str, out_path: str) -> int:
    import torch

    g = _load_gen(gen_path)
    dev = torch.device("cuda", 0)
    out: dict[str, np.ndarray] = {}

    # ---- fa_forward, non-causal, fp16 ------------------------------------------------------
    B, S, H, D = 1, 256, 2, 128
    rng = np.random.default_rng(101)
    q, k, v = (rng.standard_normal((B, S, H, D)).astype(np.float16) for _ in range(3))
    kern = _compile(g, g.fa_forward(B, S, H, D, 64, 64, 2, 128))
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    to = torch.full((B, S, H, D), float("nan"), dtype=torch.float16, device=dev)
    kern(tq, tk, tv, to)
    torch.cuda.synchronize()
    out.update({"fa.Q": q.view(np.uint16), "fa.K": k.view(np.uint16), "fa.V": v.view(np.uint16),
                "fa.Out": to.cpu().numpy().view(np.uint16),
                "fa.shape": np.array([B, S, H, D], dtype=np.int64)})

    # ---- decode_partial + decode_combine, fp16 ------------------------------------------------
    B, H, G, S, D, BN, BH, split = 1, 8, 2, 512, 128, 64, 64, 4
    rng = np.random.default_rng(102)
    q = rng.standard_normal((B, H, D)).astype(np.float16)
    k = rng.standard_normal((B, S, G, D)).astype(np.float16)
    v = rng.standard_normal((B, S, G, D)).astype(np.float16)
    part = _compile(g, g.decode_partial(B, H, G, S, D, BN, BH, split, 2))
    comb = _compile(g, g.decode_combine(B, H, D, split))
    qbuf = torch.zeros((B * H + BH) * D, dtype=torch.float16, device=dev)
    tq = qbuf[: B * H * D].view(B, H, D)
    tq.copy_(torch.from_numpy(q))
    tk, tv = torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)
    glse = torch.full((B, H, split), float("nan"), dtype=torch.float16, device=dev)
    opart = torch.full((B, H, split, D), float("nan"), dtype=torch.float16, device=dev)
    o = torch.full((B, H, D), float("nan"), dtype=torch.float16, device=dev)
    part(tq, tk, tv, glse, opart)
    comb(glse, opart, o)
    torch.cuda.synchronize()
    out.update({"dec.Q": q.view(np.uint16), "dec.K": k.view(np.uint16),
                "dec.V": v.view(np.uint16), "dec.glse": glse.cpu().numpy().view(np.uint16),
                "dec.Opart": opart.cpu().numpy().view(np.uint16),
                "dec.Out": o.cpu().numpy().view(np.uint16),
                "dec.shape": np.array([B, H, G, S, D, split], dtype=np.int64)})

    # ---- fp8gemm, unscaled e4m3 -> fp16 ---------------------------------------------------------
    M = N = K = 256
    g.SHAPE.update({"M": M, "N": N, "K": K})
    rng = np.random.default_rng(103)
    a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.float8_e4m3fn)
    b = torch.from_numpy(rng.standard_normal((N, K)).astype(np.float32)).to(torch.float8_e4m3fn)
    kern = _compile(g, g.fp8gemm(128, 128, 64, 3, 128))
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
    kern(a.to(dev), b.to(dev), c)
    torch.cuda.synchronize()
    out.update({"fp8.A": a.view(torch.uint8).numpy(), "fp8.B": b.view(torch.uint8).numpy(),
                "fp8.C": c.cpu().numpy().view(np.uint16),
                "fp8.shape": np.array([M, N, K], dtype=np.int64)})

    Path(out_path).parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, sorted(out))
    return 0


if __name__ == "__main__":
    if len(sys.argv) != 3:
        raise SystemExit("usage: python tests/golden/make_kernel_golden.py <gen.py> <out.npz>")
    sys.exit(main(sys.argv[1], sys.argv[2]))
