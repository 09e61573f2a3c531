"""The allocation-free decode entry (kta_decode_gqa_bf16_noalloc) against the regular one.

Some callers of this library cannot allocate device memory: a kernel-case harness that
allocates exactly the tensors a case declares and times a single launch (an allocation there
would synchronise the device inside the timed region), or a host whose device memory is owned
by another allocator. For them the decode partials live in a fixed array inside the library.

This test calls that entry through the C ABI, twice in a row (the array keeps the previous
call's contents; the entry must clear what has to start at zero), and compares each result
with kta_decode_gqa_bf16 called through the C ABI with a zeroed workspace of
kta_decode_workspace_bytes bytes that this test allocates, at the tolerance of the other decode
tests (|y - ref| <= 1e-2 + 1e-2 |ref|). Kept in its own file, collected last, so a run that
stops at the first failure has run every other test before it; it needs no state from them.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


def _case(lengths, hq=32, hkv=8, d=128, seed=3):
    g = torch.Generator().manual_seed(seed)
    lengths = np.asarray(lengths, dtype=np.int64)
    offsets = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int64)
    total = int(lengths.sum())
    q = torch.randn(len(lengths), hq, d, generator=g).to(torch.bfloat16)
    kc = torch.randn(total, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(total, hkv, d, generator=g).to(torch.bfloat16)
    return q, kc, vc, lengths, offsets


@pytest.mark.parametrize("lengths", [
    np.random.default_rng(0).integers(1024, 8193, size=64),  # the B=64 decode config
    [8192, 5, 700],
])
def test_noalloc_decode_matches_workspace_decode_twice(cuda_device, lengths):
    from kta_b200 import lib

    q, kc, vc, ln, off = _case(lengths)
    dev = cuda_device
    q, kc, vc = q.to(dev), kc.to(dev), vc.to(dev)
    sl = torch.as_tensor(ln, dtype=torch.int32).to(dev)
    of = torch.as_tensor(off, dtype=torch.int64).to(dev)
    max_seqlen = int(max(ln))
    bsz, hq, d = q.shape
    hkv = kc.shape[1]
    scale = d ** -0.5
    stream = int(torch.cuda.current_stream().cuda_stream)

    # the regular entry, with a workspace of its own
    need = int(lib.load().kta_decode_workspace_bytes(bsz, hq, hkv, d, max_seqlen))
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    ref = torch.full_like(q, float("nan"))
    lib.call("kta_decode_gqa_bf16", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), sl.data_ptr(),
             of.data_ptr(), ref.data_ptr(), bsz, hq, hkv, d, kc.shape[0], max_seqlen, scale,
             ws.data_ptr(), need, stream)
    torch.cuda.synchronize()
    ref_np = ref.double().cpu().numpy()
    assert np.isfinite(ref_np).all()

    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        lib.call("kta_decode_gqa_bf16_noalloc", q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                 sl.data_ptr(), of.data_ptr(), out.data_ptr(), bsz, hq, hkv, d, kc.shape[0],
                 max_seqlen, scale, stream)
        torch.cuda.synchronize()
        y = out.double().cpu().numpy()
        assert np.isfinite(y).all()
        err = np.abs(y - ref_np)
        assert np.all(err <= ATOL + RTOL * np.abs(ref_np)), f"max err {err.max():.3e}"
    assert lib.device_status(clear=True)[0] == 0


def test_noalloc_decode_rejects_a_workspace_beyond_its_array(cuda_device):
    """A call whose partials would not fit in the fixed array is refused up front, on the
    host, before any device memory is touched (the pointers here are never dereferenced)."""
    from kta_b200 import lib

    # 2048 sequences x 1024 KV heads need 8 MiB of arrival counters alone.
    status = lib.load().kta_decode_gqa_bf16_noalloc(16, 16, 16, 16, 16, 16, 2048, 1024, 1024,
                                                     128, 1024, 64, 0.1, None)
    assert status == 2  # KTA_ERR_UNSUPPORTED
