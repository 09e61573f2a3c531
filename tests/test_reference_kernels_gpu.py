"""libkta_b200 against the outputs of the reference's own kernels (tests/golden/kernels.npz:
KTA's TileLang test-set kernels run on a B200 by tests/golden/make_kernel_golden.py), on the
same inputs. The reference kernels compute in f16 where these compute in bf16, so the inputs
are rounded to bf16 first and the bound is the cases' bf16 tolerance, |y - ref| <= 1e-2 +
1e-2 |ref| (2e-2 relative for FP8):

- FP8: KTA's fp8gemm is the unscaled e4m3 GEMM (perfmodel/testset/gen.py:306-329), the
  block-scaled entry with every scale 1; the e4m3 codes are identical, so only the output
  rounding (bf16 here, f16 there) separates them;
- decode: KTA's decode_partial + decode_combine (gen.py:493-590), one sequence of 512 keys,
  8 query heads over 2 KV heads;
- attention: KTA's fa_forward (gen.py:417-486) is non-causal; under the causal mask the last
  query row of every head still sees every key, so that row must agree.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import numerics

pytestmark = pytest.mark.gpu
KZ = Path(__file__).resolve().parent / "golden" / "kernels.npz"


@pytest.fixture(scope="module")
def kz():
    return np.load(KZ)


def _f16(z, name):
    return numerics.f16_bits_to_f64(np.asarray(z[name]))


def _bf16(x: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).to(dev)


def test_fp8_matches_the_reference_fp8gemm(cuda_device, kz):
    from kta_b200 import ops

    m, n, k = (int(x) for x in kz["fp8.shape"])
    a = torch.from_numpy(np.asarray(kz["fp8.A"]).reshape(m, k)).view(torch.float8_e4m3fn)
    b = torch.from_numpy(np.asarray(kz["fp8.B"]).reshape(n, k)).view(torch.float8_e4m3fn)
    kb, nb = -(-k // 128), -(-n // 128)
    sa = torch.ones(m, kb, dtype=torch.float32, device=cuda_device)
    sb = torch.ones(nb, kb, dtype=torch.float32, device=cuda_device)
    c = ops.gemm_fp8_blockscaled(a.to(cuda_device), sa, b.to(cuda_device), sb)
    torch.cuda.synchronize()
    ref = _f16(kz, "fp8.C").reshape(m, n)
    y = c.double().cpu().numpy()
    err = np.abs(y - ref)
    assert np.all(err <= 2e-2 * np.abs(ref) + 2e-2), err.max()


def test_decode_matches_the_reference_split_and_combine(cuda_device, kz):
    from kta_b200 import ops

    b, hq, hkv, s, d, _ = (int(x) for x in kz["dec.shape"])
    q = _bf16(_f16(kz, "dec.Q").reshape(b, hq, d), cuda_device)
    kc = _bf16(_f16(kz, "dec.K").reshape(b * s, hkv, d), cuda_device)
    vc = _bf16(_f16(kz, "dec.V").reshape(b * s, hkv, d), cuda_device)
    sl = torch.tensor([s], dtype=torch.int32, device=cuda_device)
    off = torch.tensor([0], dtype=torch.int64, device=cuda_device)
    ws = torch.zeros(ops.decode_workspace_bytes(b, hq, hkv, d, s), dtype=torch.uint8,
                     device=cuda_device)
    o = ops.decode_gqa(q, kc, vc, sl, off, s, workspace=ws)
    torch.cuda.synchronize()
    ref = _f16(kz, "dec.Out").reshape(b, hq, d)
    err = np.abs(o.double().cpu().numpy() - ref)
    assert np.all(err <= 1e-2 + 1e-2 * np.abs(ref)), err.max()


def test_attention_last_rows_match_the_reference_fa_forward(cuda_device, kz):
    from kta_b200 import ops

    b, s, h, d = (int(x) for x in kz["fa.shape"])
    q, k, v = (_bf16(_f16(kz, n).reshape(b, s, h, d), cuda_device)
               for n in ("fa.Q", "fa.K", "fa.V"))
    o, _ = ops.attn_fwd_causal(q, k, v)
    torch.cuda.synchronize()
    ref = _f16(kz, "fa.Out").reshape(b, s, h, d)[:, -1]
    y = o[:, -1].double().cpu().numpy()
    err = np.abs(y - ref)
    assert np.all(err <= 1e-2 + 1e-2 * np.abs(ref)), err.max()
