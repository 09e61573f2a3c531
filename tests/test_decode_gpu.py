"""GQA decode parity on the GPU against the FP64 oracle on identical bf16 inputs, through both
C-ABI entries: kta_decode_gqa_bf16 with a caller workspace ("workspace") and
kta_decode_gqa_bf16_noalloc, whose partials live in the library's fixed array ("noalloc").
Tolerance |y - ref| <= 1e-2 + 1e-2 |ref| (bf16 output)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


def _make(lengths, hq=32, hkv=8, d=128, seed=0, gap=0):
    g = torch.Generator().manual_seed(seed)
    lengths = np.asarray(lengths, dtype=np.int64)
    offsets = np.concatenate([[0], np.cumsum(lengths + gap)[:-1]]).astype(np.int64)
    total = int(offsets[-1] + lengths[-1] + gap) if len(lengths) else 1
    total = max(total, 1)
    q = torch.randn(len(lengths), hq, d, generator=g).to(torch.bfloat16)
    kc = torch.randn(total, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(total, hkv, d, generator=g).to(torch.bfloat16)
    return q, kc, vc, lengths, offsets


ENTRIES = ["workspace", "noalloc"]


def _run(dev, q, kc, vc, lengths, offsets, max_seqlen, workspace=None, entry="noalloc"):
    """One decode through the C ABI. ``entry`` "workspace" passes a zeroed caller workspace
    of kta_decode_workspace_bytes (kta_decode_gqa_bf16); "noalloc" passes none, which
    ops.decode_gqa sends to kta_decode_gqa_bf16_noalloc when the partials fit its array."""
    from kta_b200 import ops

    bsz, hq, d = q.shape
    if workspace is None and entry == "workspace":
        need = ops.decode_workspace_bytes(bsz, hq, kc.shape[1], d, max_seqlen)
        workspace = torch.zeros(max(need, 1), dtype=torch.uint8, device=dev)
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=dev)
    ops.decode_gqa(q.to(dev), kc.to(dev), vc.to(dev),
                   torch.as_tensor(lengths, dtype=torch.int32).to(dev),
                   torch.as_tensor(offsets, dtype=torch.int64).to(dev), max_seqlen,
                   out=out, workspace=workspace)
    torch.cuda.synchronize()
    return out


def _check(out, q, kc, vc, lengths, offsets):
    d = q.shape[-1]
    ref = oatt.decode_gqa(q.double().numpy(), kc.double().numpy(), vc.double().numpy(),
                          lengths, offsets, d ** -0.5)
    y = out.double().cpu().numpy()
    err = np.abs(y - ref)
    bad = err > ATOL + RTOL * np.abs(ref)
    assert np.isfinite(y).all()
    assert not bad.any(), f"{int(bad.sum())} mismatches, max err {err.max():.3e}"


@pytest.mark.parametrize("entry", ENTRIES)
@pytest.mark.parametrize("lengths", [[1], [7, 128, 129], [512, 513, 1024, 1025],
                                     [100, 2000, 4096, 3333, 1, 640]])
def test_decode_small(cuda_device, lengths, entry):
    q, kc, vc, ln, off = _make(lengths)
    out = _run(cuda_device, q, kc, vc, ln, off, max(lengths), entry=entry)
    _check(out, q, kc, vc, ln, off)


@pytest.mark.parametrize("entry", ENTRIES)
@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (32, 4), (64, 4), (4, 1)])
def test_decode_group_sizes(cuda_device, hq, hkv, entry):
    q, kc, vc, ln, off = _make([300, 1500, 77], hq=hq, hkv=hkv)
    out = _run(cuda_device, q, kc, vc, ln, off, 2048, entry=entry)
    _check(out, q, kc, vc, ln, off)


@pytest.mark.parametrize("entry", ENTRIES)
@pytest.mark.parametrize("lengths", [[8192], [300], [8192, 8192, 17], [1] * 40])
def test_decode_splits_across_ctas(cuda_device, lengths, entry):
    """One long sequence spread over many CTAs (its pairs split and combined), and fewer
    tiles than CTAs (CTAs with empty ranges must not be counted as contributors)."""
    q, kc, vc, ln, off = _make(lengths)
    out = _run(cuda_device, q, kc, vc, ln, off, max(lengths), entry=entry)
    _check(out, q, kc, vc, ln, off)


@pytest.mark.parametrize("entry", ENTRIES)
def test_decode_one_rank_of_eight(cuda_device, entry):
    """The first 8 of the benchmark's 64 lengths U[1024, 8192] (one GPU's share at eight GPUs): each
    CTA holds about 12 tiles, so a long sequence's pair is split over five to seven CTAs and
    the last one combines more than four pieces."""
    lengths = np.random.default_rng(0).integers(1024, 8193, size=64)[:8]
    q, kc, vc, ln, off = _make(lengths, seed=8)
    out = _run(cuda_device, q, kc, vc, ln, off, 8192, entry=entry)
    _check(out, q, kc, vc, ln, off)


@pytest.mark.parametrize("entry", ENTRIES)
def test_decode_gaps_between_sequences(cuda_device, entry):
    """Sequences need not be packed back to back: rows between them are never read."""
    q, kc, vc, ln, off = _make([700, 513, 2], gap=37)
    out = _run(cuda_device, q, kc, vc, ln, off, 1024, entry=entry)
    _check(out, q, kc, vc, ln, off)


@pytest.mark.parametrize("entry", ENTRIES)
def test_decode_baseline_config(cuda_device, entry):
    """B=64, Hq=32, Hkv=8, D=128, lengths uniform in [1024, 8192] from seed 0."""
    lengths = np.random.default_rng(0).integers(1024, 8193, size=64)
    q, kc, vc, ln, off = _make(lengths)
    out = _run(cuda_device, q, kc, vc, ln, off, 8192, entry=entry)
    _check(out, q, kc, vc, ln, off)


def test_decode_workspace_reuse_is_exact(cuda_device):
    """Counters are left at zero: a second call on the same workspace gives the same bytes."""
    from kta_b200 import ops

    q, kc, vc, ln, off = _make([1500, 3000, 9])
    ws = torch.zeros(ops.decode_workspace_bytes(3, 32, 8, 128, 4096), dtype=torch.uint8,
                     device=cuda_device)
    a = _run(cuda_device, q, kc, vc, ln, off, 4096, workspace=ws)
    b = _run(cuda_device, q, kc, vc, ln, off, 4096, workspace=ws)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert int(ws[: 3 * 8 * 4].view(torch.int32).abs().sum()) == 0


def test_decode_zero_length_sequence_gives_zeros(cuda_device):
    q, kc, vc, ln, off = _make([0, 50, 0])
    out = _run(cuda_device, q, kc, vc, ln, off, 64)
    assert torch.count_nonzero(out[0].float()) == 0 and torch.count_nonzero(out[2].float()) == 0
    _check(out, q, kc, vc, ln, off)


def test_decode_rejects_length_beyond_max_on_device(cuda_device):
    """A device-side length above max_seqlen is refused by the kernel's own bounds check:
    that sequence's output is zero and the status block records KTA_ERR_DEVICE_BOUNDS."""
    from kta_b200 import lib

    lib.device_status(clear=True)
    q, kc, vc, ln, off = _make([100, 300])
    out = _run(cuda_device, q, kc, vc, ln, off, 200)  # 300 > max_seqlen
    status = lib.device_status(clear=True)
    assert status[0] == 9  # KTA_ERR_DEVICE_BOUNDS
    assert torch.count_nonzero(out[1].float()) == 0
    ref = oatt.decode_gqa(q.double().numpy(), kc.double().numpy(), vc.double().numpy(),
                          ln, off, 128 ** -0.5)
    y = out.double().cpu().numpy()
    assert np.all(np.abs(y[0] - ref[0]) <= ATOL + RTOL * np.abs(ref[0]))
