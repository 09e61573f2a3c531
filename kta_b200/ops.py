"""Tensor-level wrappers over the C ABI (include/kta_b200.h) for torch CUDA tensors.

Each function validates dtypes, shapes and devices, allocates the output with torch when
none is given (torch is the caller's allocator here, the library allocates nothing), and
launches on the current torch stream. Every call goes to libkta_b200; there is no other
implementation behind these functions.
"""

from __future__ import annotations

import torch

from kta_b200 import lib


# size of the library-owned partials array behind kta_decode_gqa_bf16_noalloc
NOALLOC_BYTES = 8 << 20

def _stream() -> int:
    return int(torch.cuda.current_stream().cuda_stream)


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("libkta_b200 operates on CUDA tensors only")


def _rows_contig(t: torch.Tensor, name: str) -> None:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit column stride")


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, *,
         b_layout: str = "nk") -> torch.Tensor:
    """C = A @ B.T (``b_layout="nk"``, B is [N, K]) or C = A @ B (``"kn"``, B is [K, N]).

    A, B, C are bf16 or f16 (all the same), row-major with unit column stride."""
    _need_cuda(a, b)
    _rows_contig(a, "A")
    _rows_contig(b, "B")
    if a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("A and B must both be bf16 or both f16")
    m, k = a.shape
    if b_layout == "nk":
        n, kb = b.shape
    elif b_layout == "kn":
        kb, n = b.shape
    else:
        raise ValueError("b_layout must be 'nk' or 'kn'")
    if kb != k:
        raise ValueError(f"K mismatch: A has {k}, B has {kb}")
    if out is None:
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    _rows_contig(out, "C")
    if out.dtype != a.dtype or tuple(out.shape) != (m, n):
        raise ValueError("C must match A's dtype and be [M, N]")
    bf16 = a.dtype == torch.bfloat16
    entry = {
        ("nk", True): "kta_gemm_bf16",
        ("nk", False): "kta_gemm_f16",
        ("kn", True): "kta_gemm_nn_bf16",
        ("kn", False): "kta_gemm_nn_f16",
    }[(b_layout, bf16)]
    lib.call(entry, a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
             a.stride(0), b.stride(0), out.stride(0), _stream())
    return out


def gemm_fp8_blockscaled(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    """C (bf16) = dequant(A, sa) @ dequant(B, sb).T with per-1x128 activation scales sa
    [M, ceil(K/128)] and per-128x128 weight scales sb [ceil(N/128), ceil(K/128)] (fp32)."""
    _need_cuda(a, sa, b, sb)
    if a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn:
        raise ValueError("A and B must be float8_e4m3fn")
    if sa.dtype != torch.float32 or sb.dtype != torch.float32:
        raise ValueError("scales must be float32")
    for t, name in ((a, "A"), (b, "B"), (sa, "sa"), (sb, "sb")):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    m, k = a.shape
    n, kb = b.shape
    if kb != k:
        raise ValueError("K mismatch")
    kblk, nblk = -(-k // 128), -(-n // 128)
    if tuple(sa.shape) != (m, kblk) or tuple(sb.shape) != (nblk, kblk):
        raise ValueError(f"scales must be sa [{m}, {kblk}] and sb [{nblk}, {kblk}]")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or not out.is_contiguous():
        raise ValueError("C must be a contiguous bf16 [M, N] tensor")
    lib.call("kta_gemm_fp8_blockscaled", a.data_ptr(), sa.data_ptr(), b.data_ptr(),
             sb.data_ptr(), out.data_ptr(), m, n, k, _stream())
    return out


def gemm_4bit(a: torch.Tensor, bq: torch.Tensor, sc: torch.Tensor, fmt: str = "int4",
              group: int = 32, out: torch.Tensor | None = None) -> torch.Tensor:
    """C = A @ B^T with B dequantised from 4-bit codes: A f16 [M, K]; Bq int8/uint8 [N, K/2]
    (two codes per byte, the lower nibble first); Sc f16 [N, K/group]. ``fmt`` "int4"
    (value = code - 8, any power-of-two group >= 16) or "e2m1" (NVFP4, group 16)."""
    _need_cuda(a, bq, sc)
    if a.dtype != torch.float16 or sc.dtype != torch.float16:
        raise ValueError("A and Sc must be f16")
    if bq.dtype not in (torch.int8, torch.uint8):
        raise ValueError("Bq must be int8 or uint8 bytes")
    for t, name in ((a, "A"), (bq, "Bq"), (sc, "Sc")):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    m, k = a.shape
    n = bq.shape[0]
    if bq.shape != (n, k // 2) or sc.shape != (n, k // group):
        raise ValueError("Bq must be [N, K/2] and Sc [N, K/group]")
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16, device=a.device)
    if fmt == "int4":
        lib.call("kta_gemm_w4a16_f16", a.data_ptr(), bq.data_ptr(), sc.data_ptr(),
                 out.data_ptr(), m, n, k, group, _stream())
    elif fmt == "e2m1":
        if group != 16:
            raise ValueError("NVFP4 scales one block of 16 elements")
        lib.call("kta_gemm_nvfp4_f16", a.data_ptr(), bq.data_ptr(), sc.data_ptr(),
                 out.data_ptr(), m, n, k, _stream())
    else:
        raise ValueError(f"unknown 4-bit format {fmt!r}")
    return out


def moe_gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """MoE expert GEMM: A [T, K] with tokens grouped by expert (T / E rows each, a multiple
    of 128), W [E, K, N]; C[rows of e] = A[rows of e] @ W[e]; f16 or bf16, fp32 accumulate."""
    _need_cuda(a, w)
    if a.dim() != 2 or w.dim() != 3 or a.shape[1] != w.shape[1]:
        raise ValueError("A must be [T, K] and W [E, K, N]")
    if a.dtype != w.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("A and W must share an f16 or bf16 dtype")
    if not a.is_contiguous() or not w.is_contiguous():
        raise ValueError("A and W must be contiguous")
    t, k = a.shape
    e, _, n = w.shape
    if out is None:
        out = torch.empty((t, n), dtype=a.dtype, device=a.device)
    entry = "kta_moe_gemm_f16" if a.dtype == torch.float16 else "kta_moe_gemm_bf16"
    lib.call(entry, a.data_ptr(), w.data_ptr(), out.data_ptr(), e, t, n, k, _stream())
    return out


def _rowop_check(x: torch.Tensor, name: str) -> None:
    if x.dim() != 2 or not x.is_contiguous():
        raise ValueError(f"{name} must be a contiguous [M, N] tensor")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"{name} must be f16 or bf16")


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """Y = X * rsqrt(mean(X^2, -1) + eps) * W over the rows of X [M, N] (f16 or bf16), W [N]
    of the same dtype; fp32 statistics."""
    _need_cuda(x, w)
    _rowop_check(x, "X")
    if w.dtype != x.dtype or w.shape != (x.shape[1],) or not w.is_contiguous():
        raise ValueError("W must be a contiguous [N] tensor of X's dtype")
    if out is None:
        out = torch.empty_like(x)
    entry = "kta_rmsnorm_f16" if x.dtype == torch.float16 else "kta_rmsnorm_bf16"
    lib.call(entry, x.data_ptr(), w.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1],
             float(eps), _stream())
    return out


def softmax(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Row softmax of X [M, N] (f16 or bf16), fp32 max and sum."""
    _need_cuda(x)
    _rowop_check(x, "X")
    if out is None:
        out = torch.empty_like(x)
    entry = "kta_softmax_f16" if x.dtype == torch.float16 else "kta_softmax_bf16"
    lib.call(entry, x.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], _stream())
    return out


def attn_fwd_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                    out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """Causal attention forward. Q, K, V bf16 [B, S, H, D] contiguous; returns O bf16
    [B, S, H, D] and LSE fp32 [B, H, S] (natural log)."""
    _need_cuda(q, k, v)
    for t, name in ((q, "Q"), (k, "K"), (v, "V")):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.dim() != 4:
            raise ValueError(f"{name} must be a contiguous bf16 [B, S, H, D] tensor")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("Q, K, V must have the same shape")
    bsz, s, h, d = q.shape
    if scale is None:
        scale = d ** -0.5
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((bsz, h, s), dtype=torch.float32, device=q.device)
    if out.shape != q.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("O must be a contiguous bf16 tensor shaped like Q")
    if tuple(lse.shape) != (bsz, h, s) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("LSE must be a contiguous fp32 [B, H, S] tensor")
    lib.call("kta_attn_fwd_causal_bf16", q.data_ptr(), k.data_ptr(), v.data_ptr(),
             out.data_ptr(), lse.data_ptr(), bsz, h, s, d, float(scale), _stream())
    return out, lse


def decode_workspace_bytes(batch: int, hq: int, hkv: int, d: int, max_seqlen: int) -> int:
    return int(lib.load().kta_decode_workspace_bytes(batch, hq, hkv, d, max_seqlen))


def decode_gqa(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
               seqlens: torch.Tensor, kv_offsets: torch.Tensor, max_seqlen: int,
               scale: float | None = None, out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """GQA decode: Q bf16 [B, Hq, D]; caches bf16 [T, Hkv, D] with sequence b at rows
    kv_offsets[b] .. kv_offsets[b] + seqlens[b]; seqlens int32 [B], kv_offsets int64 [B].
    ``workspace`` (uint8, zero-initialised once) may be reused across calls on one stream.
    Without one, the library's own 8 MiB array is used when the split partials fit
    (kta_decode_gqa_bf16_noalloc: no allocation; the entry clears the array's arrival
    counters with a memset on the stream before its kernel; calls that overlap on the GPU
    share the array, so concurrent streams must pass their own workspace)."""
    _need_cuda(q, k_cache, v_cache, seqlens, kv_offsets)
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or \
            v_cache.dtype != torch.bfloat16:
        raise ValueError("Q and the caches must be bf16")
    for t, name in ((q, "Q"), (k_cache, "K cache"), (v_cache, "V cache")):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if seqlens.dtype != torch.int32 or kv_offsets.dtype != torch.int64:
        raise ValueError("seqlens must be int32 and kv_offsets int64")
    bsz, hq, d = q.shape
    hkv = k_cache.shape[1]
    if k_cache.shape != v_cache.shape or k_cache.shape[2] != d:
        raise ValueError("K and V caches must be [T, Hkv, D] with Q's D")
    if scale is None:
        scale = d ** -0.5
    if out is None:
        out = torch.empty_like(q)
    need = decode_workspace_bytes(bsz, hq, hkv, d, max_seqlen)
    if workspace is None and need <= NOALLOC_BYTES:
        lib.call("kta_decode_gqa_bf16_noalloc", q.data_ptr(), k_cache.data_ptr(),
                 v_cache.data_ptr(), seqlens.data_ptr(), kv_offsets.data_ptr(), out.data_ptr(),
                 bsz, hq, hkv, d, k_cache.shape[0], int(max_seqlen), float(scale), _stream())
        return out
    if workspace is None:
        workspace = torch.zeros(max(need, 1), dtype=torch.uint8, device=q.device)
    if workspace.numel() < need:
        raise ValueError(f"workspace needs {need} bytes")
    lib.call("kta_decode_gqa_bf16", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
             seqlens.data_ptr(), kv_offsets.data_ptr(), out.data_ptr(), bsz, hq, hkv, d,
             k_cache.shape[0], int(max_seqlen), float(scale), workspace.data_ptr(),
             workspace.numel(), _stream())
    return out


class _HostPipe:
    """Device buffers and streams of one host-buffer GEMM shape for one caller stream, kept
    across calls. ``done`` marks the end of the last call's read-back: the next call's
    uploads wait for it before they overwrite A and B, so a later call never changes the
    buffers of one still in flight."""

    def __init__(self, m: int, n: int, k: int, dtype: torch.dtype, device: torch.device) -> None:
        self.a = torch.empty((m, k), dtype=dtype, device=device)
        self.b = torch.empty((n, k), dtype=dtype, device=device)
        self.c = torch.empty((m, n), dtype=dtype, device=device)
        self.h2d = torch.cuda.Stream(device=device)
        self.comp = torch.cuda.Stream(device=device)
        self.d2h = torch.cuda.Stream(device=device)
        self.done: torch.cuda.Event | None = None


_PIPES: dict[tuple, _HostPipe] = {}


def gemm_host(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
              chunks: int = 2, device: torch.device | None = None,
              wait: bool = True) -> torch.Tensor:
    """C = A @ B.T with A, B and C in (pinned) host memory, end to end.

    The call copies B to the device, then A in ``chunks`` row blocks; each block's GEMM
    starts as soon as its rows have landed, and each block of C is copied back as soon as it
    is computed, on three streams, so host-device traffic in both directions overlaps the
    tensor-core work. The work is ordered after what the caller's current stream has queued,
    and the caller's stream is ordered after the read-back.

    With ``wait`` (the default) the call returns once C is complete on the host. With
    ``wait=False`` it returns as soon as the work is queued: C is valid on the host once the
    caller's current stream has reached this point (synchronise it, or an event recorded on
    it), and A and B must stay unchanged until then.

    Two blocks by default: at 8192^3 two pipelines in flight ran 207.9 / 206.6 / 200.4 / 188.3
    TFLOP/s end to end with 2 / 4 / 8 / 16 blocks, the PCIe link being the bound and each
    smaller block's GEMM leaving a wave of tiles partly empty on the path to its read-back.

    Device buffers are kept per (shape, dtype, device, caller stream), so calls from
    different streams never share them; consecutive calls from one stream reuse them in
    order (each call's uploads wait for the previous call's read-back)."""
    if a.is_cuda or b.is_cuda:
        raise ValueError("gemm_host takes host tensors")
    m, k = a.shape
    n, kb = b.shape
    if kb != k or a.dtype != b.dtype:
        raise ValueError("A [M, K] and B [N, K] of one dtype")
    device = device or torch.device("cuda", torch.cuda.current_device())
    caller = torch.cuda.current_stream(device)
    key = (m, n, k, a.dtype, device, caller.cuda_stream)
    pipe = _PIPES.get(key)
    if pipe is None:
        pipe = _PIPES[key] = _HostPipe(m, n, k, a.dtype, device)
    if out is None:
        out = torch.empty((m, n), dtype=a.dtype, pin_memory=True)
    chunks = max(1, min(chunks, -(-m // 128)))
    rows = -(-m // chunks)
    rows = -(-rows // 128) * 128
    pipe.h2d.wait_stream(caller)
    if pipe.done is not None:
        pipe.h2d.wait_event(pipe.done)
    with torch.cuda.stream(pipe.h2d):
        pipe.b.copy_(b, non_blocking=True)
        b_ready = torch.cuda.Event()
        b_ready.record(pipe.h2d)
        a_ready = []
        for r0 in range(0, m, rows):
            pipe.a[r0:r0 + rows].copy_(a[r0:r0 + rows], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(pipe.h2d)
            a_ready.append(ev)
    c_ready = []
    with torch.cuda.stream(pipe.comp):
        pipe.comp.wait_event(b_ready)
        for i, r0 in enumerate(range(0, m, rows)):
            pipe.comp.wait_event(a_ready[i])
            gemm(pipe.a[r0:r0 + rows], pipe.b, out=pipe.c[r0:r0 + rows])
            ev = torch.cuda.Event()
            ev.record(pipe.comp)
            c_ready.append(ev)
    with torch.cuda.stream(pipe.d2h):
        for i, r0 in enumerate(range(0, m, rows)):
            pipe.d2h.wait_event(c_ready[i])
            out[r0:r0 + rows].copy_(pipe.c[r0:r0 + rows], non_blocking=True)
        pipe.done = torch.cuda.Event()
        pipe.done.record(pipe.d2h)
    caller.wait_event(pipe.done)
    if wait:
        pipe.done.synchronize()
    return out
