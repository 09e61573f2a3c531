"""Seeded input generation for the B200 cases (measurement and checks).

Mirrors src/kta/measure/inputs.py:22-93 and src/kta/checks/inputs.py:16-48: tensor shapes
are expressions over the shape variables, distributions form an open table whose generators
take ``(dims, dtype, numpy Generator)``, and every draw starts from a ``random.Random``
stream: ``np.random.default_rng(rng.getrandbits(63))`` (inputs.py:90), with streams named
as the reference's ``ctx.rng(name)`` derives them (src/kta/core/context.py:74-77).

B200 additions (deliberate; the reference's table is open by design, checks/inputs.py:3-4):
- host dtypes ``bf16`` (carried as uint16 bit patterns; the reference has none yet,
  measure/inputs.py:40-43) and ``e4m3`` (uint8 patterns);
- ``normal_scaled``: N(0,1)/sqrt(last dim), the GEMM cases' N(0,1)/sqrt(K);
- ``outliers``: N(0,1) with 1% of entries multiplied by 20 (the FP8 case's source values).

``quantize_blockwise_e4m3`` turns float source values into e4m3 codes with fp32 block
scales amax/448 (per 1x128 for activations, per 128x128 for weights).
"""

from __future__ import annotations

import hashlib
import random
from collections.abc import Callable
from typing import Any

import numpy as np

from kta_b200.expr import Expr
from kta_b200.schemas import TensorSpec


class NotSupported(ValueError):
    pass


# storage dtype of each case dtype (bf16 and e4m3 travel as raw bit patterns)
DTYPES: dict[str, Any] = {
    "f16": np.float16,
    "float16": np.float16,
    "bf16": np.uint16,
    "bfloat16": np.uint16,
    "e4m3": np.uint8,
    "f32": np.float32,
    "float32": np.float32,
    "f64": np.float64,
    "float64": np.float64,
    "i32": np.int32,
    "int32": np.int32,
    "i64": np.int64,
    "int64": np.int64,
    "i8": np.int8,
    "int8": np.int8,
}
ITEMSIZE = {k: np.dtype(v).itemsize for k, v in DTYPES.items()}
EXTREME_SCALE = {"f16": 16.0, "float16": 16.0, "bf16": 16.0, "bfloat16": 16.0,
                 "f32": 1e3, "float32": 1e3}
EXTREME_FRACTION = 0.01
OUTLIER_FRACTION = 0.01
OUTLIER_SCALE = 20.0
E4M3_MAX = 448.0

Generator = Callable[[tuple[int, ...], str, np.random.Generator], np.ndarray]


def np_dtype(dtype: str) -> Any:
    if dtype not in DTYPES:
        raise NotSupported(f"dtype {dtype!r} has no host representation")
    return DTYPES[dtype]


def dims(spec: TensorSpec, shape: dict[str, Any]) -> tuple[int, ...]:
    return tuple(int(Expr.parse(d, set(shape)).eval(shape)) for d in spec.shape)


def nbytes(spec: TensorSpec, shape: dict[str, Any]) -> int:
    return int(np.prod(dims(spec, shape), dtype=np.int64)) * ITEMSIZE[spec.dtype]


def named_rng(seed: int, name: str) -> random.Random:
    """The stream ``name`` of context seed ``seed``."""
    digest = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return random.Random(int.from_bytes(digest[:8], "big"))


# ---- distributions ---------------------------------------------------------------------

def _normal(d, dtype, g):
    return g.standard_normal(d)


def _zeros(d, dtype, g):
    return np.zeros(d)


def _uniform(d, dtype, g):
    return g.uniform(-1.0, 1.0, d)


def _extreme(d, dtype, g):
    x = g.standard_normal(d)
    mask = g.random(d) < EXTREME_FRACTION
    return np.where(mask, x * EXTREME_SCALE.get(dtype, 1e3), x)


def _cancellation(d, dtype, g):
    x = g.standard_normal(d) * 8.0
    flat = x.reshape(-1)
    n = flat.size - flat.size % 2
    flat[1:n:2] = -flat[0:n:2] + g.standard_normal(n // 2) * 1e-2
    return x


def _dominant_tail(d, dtype, g):
    x = g.standard_normal(d)
    if len(d) > 0 and d[-1] > 0:
        x[..., -1] = 8.0
    return x


def _large_dynamic_range(d, dtype, g):
    sign = np.where(g.random(d) < 0.5, -1.0, 1.0)
    return sign * np.exp2(g.uniform(-6.0, 3.0, d))


def _normal_scaled(d, dtype, g):
    k = d[-1] if len(d) else 1
    return g.standard_normal(d) / np.sqrt(max(k, 1))


def _outliers(d, dtype, g):
    x = g.standard_normal(d)
    mask = g.random(d) < OUTLIER_FRACTION
    return np.where(mask, x * OUTLIER_SCALE, x)


BASE: dict[str, Generator] = {
    "normal": _normal,
    "zeros": _zeros,
    "uniform": _uniform,
    "extreme": _extreme,
}
TABLE: dict[str, Generator] = {
    **BASE,
    "cancellation": _cancellation,
    "dominant_tail": _dominant_tail,
    "large_dynamic_range": _large_dynamic_range,
    "normal_scaled": _normal_scaled,
    "outliers": _outliers,
}


# ---- casts -----------------------------------------------------------------------------

def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float64 -> bf16 bit patterns: f64 -> f32 (nearest), then f32 -> bf16 nearest-even."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    out = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)
    return np.where(np.isnan(f), np.uint16(0x7FC0), out)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def cast(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype in ("bf16", "bfloat16"):
        return to_bf16_bits(x)
    if dtype == "e4m3":
        raise NotSupported("e4m3 tensors come from quantize_blockwise_e4m3, not a plain cast")
    return np.ascontiguousarray(x).astype(np_dtype(dtype))


def generate(spec: TensorSpec, shape: dict[str, Any], dist: str, rng: random.Random,
             table: dict[str, Generator] | None = None) -> np.ndarray:
    gens = table if table is not None else TABLE
    if dist not in gens:
        raise NotSupported(f"input distribution {dist!r} (known: {sorted(gens)})")
    g = np.random.default_rng(rng.getrandbits(63))
    return cast(np.ascontiguousarray(gens[dist](dims(spec, shape), spec.dtype, g)), spec.dtype)


def random_inputs(problem, shape: dict[str, Any], dist: str, rng: random.Random,
                  table: dict[str, Generator] | None = None) -> dict[str, np.ndarray]:
    """One input set: every input tensor of ``problem`` (src/kta/measure/jobs.py:120-123)."""
    return {t.name: generate(t, shape, dist, rng, table) for t in problem.inputs}


# ---- block-scaled e4m3 -------------------------------------------------------------------

def quantize_blockwise_e4m3(x: np.ndarray, block_rows: int, block_cols: int = 128
                            ) -> tuple[np.ndarray, np.ndarray]:
    """e4m3 codes and fp32 scales of a 2-D float array, one scale per
    ``block_rows x block_cols`` block: scale = amax / 448 (1 for an all-zero block),
    code = e4m3(x / scale) rounded to nearest even (torch's float8_e4m3fn cast)."""
    import torch

    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    rb, cb = -(-rows // block_rows), -(-cols // block_cols)
    pad = np.zeros((rb * block_rows, cb * block_cols), dtype=np.float32)
    pad[:rows, :cols] = x
    blocks = pad.reshape(rb, block_rows, cb, block_cols)
    amax = np.abs(blocks).max(axis=(1, 3))
    scale = np.where(amax > 0, amax / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)
    q = blocks / scale[:, None, :, None]
    q = q.reshape(rb * block_rows, cb * block_cols)[:rows, :cols]
    codes = torch.from_numpy(np.ascontiguousarray(q)).to(torch.float8_e4m3fn)
    return codes.view(torch.uint8).numpy().copy(), scale


# ---- 4-bit weights (w4a16 int4, NVFP4 e2m1) ------------------------------------------------

E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def quantize_4bit(x: np.ndarray, fmt: str, group: int) -> tuple[np.ndarray, np.ndarray]:
    """Packed 4-bit codes (int8 [N, K/2], two per byte, the lower nibble first) and f16 scales
    [N, K/group] of a 2-D float array. int4: scale = amax / 7 (f16), code = round(x / scale) + 8
    clipped to [0, 15] (value = code - 8); e2m1: scale = amax / 6 (f16), code = the nearest e2m1
    magnitude's index, sign in bit 3. An all-zero group gets scale 1."""
    x = np.asarray(x, dtype=np.float32)
    n, k = x.shape
    if k % group or k % 2:
        raise NotSupported(f"K={k} must be a multiple of the group ({group}) and of 2")
    blocks = x.reshape(n, k // group, group)
    amax = np.abs(blocks).max(axis=-1)
    top = 7.0 if fmt == "int4" else 6.0
    scale = np.where(amax > 0, amax / top, 1.0).astype(np.float16)
    y = blocks / scale.astype(np.float32)[..., None]
    if fmt == "int4":
        codes = np.clip(np.rint(y) + 8, 0, 15).astype(np.uint8)
    elif fmt == "e2m1":
        idx = np.abs(np.abs(y)[..., None] - E2M1_GRID).argmin(axis=-1).astype(np.uint8)
        codes = idx | np.where(y < 0, np.uint8(8), np.uint8(0))
    else:
        raise NotSupported(f"4-bit format {fmt!r}")
    codes = codes.reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed.view(np.int8), scale


# ---- whole input sets of a case -----------------------------------------------------------

def case_inputs(problem, shape: dict[str, Any], dist: str, rng: random.Random,
                table: dict[str, Generator] | None = None
                ) -> tuple[dict[str, Any], dict[str, np.ndarray]]:
    """One input set of ``problem`` at ``shape`` from the stream ``rng``: the shape with any
    derived sizes filled in, and the host arrays in input order.

    Two Problem params extend the per-tensor draw (src/kta/measure/jobs.py:120-123):
    ``lengths`` {low, high, seqlens, offsets, total} draws per-sequence lengths uniform in
    [low, high] (clipped to max_seqlen), packs them back to back and sets the total as a
    shape variable; ``quantize`` {tensor: {scale, block}} draws the tensor's source values
    from ``dist`` and stores e4m3 codes plus fp32 block scales amax/448; ``pack4`` {tensor,
    scale, format, group} draws [N, K] source values and stores packed 4-bit codes plus f16
    group scales (``quantize_4bit``)."""
    shape = dict(shape)
    out: dict[str, np.ndarray] = {}
    lengths = problem.params.get("lengths")
    if lengths:
        g = np.random.default_rng(rng.getrandbits(63))
        hi = min(int(lengths["high"]), int(shape.get("max_seqlen", lengths["high"])))
        lo = min(int(lengths["low"]), hi)
        ln = g.integers(lo, hi + 1, size=int(shape["B"])).astype(np.int32)
        off = np.concatenate([[0], np.cumsum(ln, dtype=np.int64)[:-1]]).astype(np.int64)
        shape[lengths["total"]] = int(ln.sum())
        out[lengths["seqlens"]] = ln
        out[lengths["offsets"]] = off
    quant = problem.params.get("quantize") or {}
    scale_of = {v["scale"]: k for k, v in quant.items()}
    pack4 = problem.params.get("pack4")
    if pack4:
        # the packed tensor's source values are [N, K] (the packed shape is [N, K/2])
        spec = TensorSpec(name=pack4["tensor"], shape=["N", "K"], dtype="f32",
                          layout="row_major")
        src = generate(spec, shape, dist, rng, table).astype(np.float32)
        out[pack4["tensor"]], out[pack4["scale"]] = quantize_4bit(
            src, pack4["format"], int(pack4["group"]))
    for t in problem.inputs:
        if t.name in out:
            continue
        if t.name in quant:
            spec = TensorSpec(name=t.name, shape=t.shape, dtype="f32", layout=t.layout)
            src = generate(spec, shape, dist, rng, table).astype(np.float32)
            rows = int(quant[t.name]["block"][0])
            codes, scales = quantize_blockwise_e4m3(src, rows, int(quant[t.name]["block"][1]))
            out[t.name] = codes
            out[quant[t.name]["scale"]] = scales
        elif t.name in scale_of:
            continue  # produced with its tensor
        else:
            out[t.name] = generate(t, shape, dist, rng, table)
    return shape, {t.name: out[t.name] for t in problem.inputs}
