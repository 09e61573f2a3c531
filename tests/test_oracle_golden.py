"""The oracle pinned against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from the reference's code) and against exact definitions.

CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import fp8 as ofp8
from oracle import gemm as ogemm
from oracle import numerics

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def st():
    return np.load(GOLDEN / "statements.npz")


def test_gemm_nn_matches_reference_statement_runner(st):
    """The seed cases' `C = A @ B` through the reference's ref_torch.py (FP64)."""
    a, b = st["nn.A"], st["nn.B"]
    ref = st["nn.C.f64"].reshape(a.shape[0], b.shape[1])
    np.testing.assert_allclose(ogemm.gemm_nn(a.astype(np.float64), b.astype(np.float64)), ref,
                               rtol=1e-12, atol=1e-12)


def test_gemm_tn_matches_reference_statement_runner(st):
    a, b = st["nn.A"], st["tn.B"]
    ref = st["tn.C.f64"].reshape(a.shape[0], b.shape[0])
    np.testing.assert_allclose(ogemm.gemm_tn(a.astype(np.float64), b.astype(np.float64)), ref,
                               rtol=1e-12, atol=1e-12)
    # the library run in the inputs' own dtype (f16) rounds to f16: within f16 rounding
    lib = st["tn.C.lib"].reshape(ref.shape)
    assert np.abs(lib - ref).max() <= 2e-3 * max(1.0, np.abs(ref).max())


def test_causal_attention_matches_reference_statement_runner(st):
    q, k, v = st["attn.Q"], st["attn.K"], st["attn.V"]
    bsz, s, h, d = q.shape
    o, lse = oatt.causal_fwd(q, k, v, d ** -0.5)
    np.testing.assert_allclose(o, st["attn.O.f64"].reshape(o.shape), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, st["attn.LSE.f64"].reshape(lse.shape), rtol=1e-10,
                               atol=1e-12)


def test_decode_matches_reference_statement_runner(st):
    q, kc, vc = st["dec.Q"], st["dec.Kc"], st["dec.Vc"]
    o = oatt.decode_gqa(q, kc, vc, st["dec.seqlens"], st["dec.offsets"], q.shape[-1] ** -0.5)
    np.testing.assert_allclose(o, st["dec.O.f64"].reshape(o.shape), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("chunk", [1, 4, 16, 1000])
def test_decode_split_combine_equals_closed_form(st, chunk):
    """The reference's split-KV partials (log2 LSE) + exp2 combine is the same function."""
    args = (st["dec.Q"], st["dec.Kc"], st["dec.Vc"], st["dec.seqlens"], st["dec.offsets"],
            st["dec.Q"].shape[-1] ** -0.5)
    np.testing.assert_allclose(oatt.decode_split(*args, chunk=chunk), oatt.decode_gqa(*args),
                               rtol=1e-12, atol=1e-12)


def test_fp8_statement_matches_reference_statement_runner(st):
    """The block-scaled statement, run by the reference's runner on dequantisable values."""
    a, b, sa, sb = st["fp8.A"], st["fp8.B"], st["fp8.sa"], st["fp8.sb"]
    ad = a.astype(np.float64) * np.repeat(sa.astype(np.float64), 128, axis=1)[:, :a.shape[1]]
    s = np.repeat(np.repeat(sb.astype(np.float64), 128, 0), 128, 1)[:b.shape[0], :b.shape[1]]
    ref = st["fp8.C.f64"].reshape(a.shape[0], b.shape[0])
    np.testing.assert_allclose(ad @ (b.astype(np.float64) * s).T, ref, rtol=1e-12, atol=1e-12)


def test_e4m3_table_matches_torch_float8():
    codes = torch.arange(256, dtype=torch.uint8)
    t = codes.view(torch.float8_e4m3fn).to(torch.float64).numpy()
    ours = numerics.E4M3_TABLE
    same = (ours == t) | (np.isnan(ours) & np.isnan(t))
    assert same.all()


def test_e4m3_rounding_matches_torch_cast():
    g = np.random.default_rng(0)
    x = np.concatenate([g.standard_normal(20000) * 50, g.uniform(-448, 448, 20000),
                        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 1e-6])])
    x = x.astype(np.float32).astype(np.float64)
    ours = numerics.f64_to_e4m3_bits(x)
    theirs = torch.from_numpy(x.astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8)
    assert np.array_equal(ours, theirs.numpy())


def test_fp8_quantiser_matches_product_quantiser():
    from kta_b200 import inputs as kinp

    g = np.random.default_rng(1)
    x = g.standard_normal((130, 300)) * np.where(g.random((130, 300)) < 0.01, 20, 1)
    for rows in (1, 128):
        c1, s1 = ofp8.quantize(x, rows)
        c2, s2 = kinp.quantize_blockwise_e4m3(x, rows)
        assert np.array_equal(s1, s2) and np.array_equal(c1, c2)


def test_bf16_widening_and_rounding_match_torch():
    g = np.random.default_rng(2)
    x = np.concatenate([g.standard_normal(50000) * 10, np.array([0.0, 1e-40, -3.0e38])])
    bits = numerics.f64_to_bf16_bits(x)
    t = torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
    assert np.array_equal(bits.view(np.int16), t)
    back = numerics.bf16_bits_to_f64(bits)
    assert np.array_equal(back, torch.from_numpy(t).view(torch.bfloat16).double().numpy())


def test_rmsnorm_matches_reference_statement_runner(st):
    from oracle import rowops

    x, w = st["rms.X"], st["rms.W"]
    np.testing.assert_allclose(rowops.rmsnorm(x, w, 1e-6), st["rms.Y.f64"].reshape(x.shape),
                               rtol=1e-12, atol=1e-12)


def test_softmax_matches_reference_statement_runner(st):
    from oracle import rowops

    x = st["smax.X"]
    np.testing.assert_allclose(rowops.softmax(x), st["smax.Y.f64"].reshape(x.shape),
                               rtol=1e-12, atol=1e-15)


def test_moe_matches_reference_statement_runner(st):
    a, w = st["moe.A"], st["moe.W"]
    ref = st["moe.C.f64"].reshape(a.shape[0], w.shape[2])
    np.testing.assert_allclose(ogemm.moe_gemm(a, w), ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("tag,fmt,group", [("w4", "int4", 32), ("nvfp4", "e2m1", 16)])
def test_4bit_gemm_matches_reference_statement_runner(st, tag, fmt, group):
    """The reference's statement runner in FP64 forms B in f16 (as the reference's kernels form
    B_shared) and multiplies in FP64; the oracle does the same: equal to FP64 summation order.
    Without the f16 rounding of B the product would differ (the fixture would catch a
    statement or oracle that dropped it)."""
    from oracle import dequant

    a, bq, sc = st[f"{tag}.A"], st[f"{tag}.Bq"], st[f"{tag}.Sc"]
    ref = st[f"{tag}.C.f64"].reshape(a.shape[0], bq.shape[0])
    got = dequant.gemm(a, bq, sc, fmt, group)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)
    unrounded = a.astype(np.float64) @ (dequant.decode(dequant.unpack(bq), fmt) * np.repeat(
        sc.astype(np.float64), group, axis=1)).T
    assert not np.allclose(unrounded, ref, rtol=1e-12, atol=1e-12)


def test_e2m1_decode_is_the_e2m1_table():
    from oracle import dequant

    vals = dequant.decode(np.arange(16), "e2m1")
    assert list(vals) == [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]


# ---- pins to the reference's own kernels (tests/golden/kernels.npz, made on a B200 by
# ---- tests/golden/make_kernel_golden.py from KTA's TileLang test-set kernels) -------------
@pytest.fixture(scope="module")
def kz():
    return np.load(GOLDEN / "kernels.npz")


def _f16(bits):
    return numerics.f16_bits_to_f64(np.asarray(bits))


def test_attention_oracle_matches_the_reference_fa_forward_kernel(kz):
    """KTA's fa_forward (perfmodel/testset/gen.py:417-486: online softmax in exp2 form, P in
    f16, f16 output) against the oracle's non-causal attention in FP64 on the same f16 inputs:
    within the kernel's own f16 roundings. The causal oracle differs from it by far more, so
    the pin tells the two functions apart."""
    b, s, h, d = (int(x) for x in kz["fa.shape"])
    q, k, v = (_f16(kz[n]).reshape(b, s, h, d) for n in ("fa.Q", "fa.K", "fa.V"))
    y = _f16(kz["fa.Out"]).reshape(b, s, h, d)
    o, _ = oatt.attn_fwd(q, k, v, d ** -0.5, causal=False)
    err = np.abs(y - o)
    assert np.isfinite(y).all()
    assert np.all(err <= 2e-3 + 2e-3 * np.abs(o)), err.max()
    oc, _ = oatt.attn_fwd(q, k, v, d ** -0.5, causal=True)
    assert np.abs(y - oc).max() > 0.05
    # the last query row sees every key under the causal mask too
    np.testing.assert_array_less(np.abs(y[:, -1] - oc[:, -1]), 2e-3 + 2e-3 * np.abs(oc[:, -1]))


def test_decode_oracle_matches_the_reference_split_and_combine_kernels(kz):
    """KTA's decode_partial (gen.py:493-560) and decode_combine (gen.py:563-590): the oracle's
    per-chunk partials and log2-unit LSE against the split kernel's f16 outputs, the oracle's
    combine of the kernel's own partials against the combine kernel's output, and the oracle's
    whole decode against it."""
    b, hq, hkv, s, d, split = (int(x) for x in kz["dec.shape"])
    q = _f16(kz["dec.Q"]).reshape(b, hq, d)
    k = _f16(kz["dec.K"]).reshape(b, s, hkv, d)
    v = _f16(kz["dec.V"]).reshape(b, s, hkv, d)
    glse = _f16(kz["dec.glse"]).reshape(b, hq, split)
    opart = _f16(kz["dec.Opart"]).reshape(b, hq, split, d)
    out = _f16(kz["dec.Out"]).reshape(b, hq, d)
    parts, lse2 = oatt.decode_partials(q[0], k[0], v[0], s, 0, d ** -0.5, s // split)
    assert np.all(np.abs(glse[0] - lse2) <= 1e-2 + 1e-3 * np.abs(lse2)), \
        np.abs(glse[0] - lse2).max()
    assert np.all(np.abs(opart[0] - parts) <= 2e-3 + 2e-3 * np.abs(parts)), \
        np.abs(opart[0] - parts).max()
    comb = oatt.decode_combine(opart[0], glse[0])
    assert np.all(np.abs(out[0] - comb) <= 1e-3 + 1e-3 * np.abs(comb)), np.abs(out[0] - comb).max()
    full = oatt.decode_gqa(q, k[0], v[0], np.array([s]), np.array([0]), d ** -0.5)
    assert np.all(np.abs(out - full) <= 2e-3 + 2e-3 * np.abs(full)), np.abs(out - full).max()


def test_fp8_oracle_matches_the_reference_fp8gemm_kernel(kz):
    """KTA's fp8gemm (gen.py:306-329: C = A B^T in e4m3, fp32 accumulate, f16 out) against the
    oracle's block-scaled statement with every scale 1 (the unscaled special case), on the same
    codes: within the f16 rounding of C."""
    m, n, kk = (int(x) for x in kz["fp8.shape"])
    a = np.asarray(kz["fp8.A"]).reshape(m, kk)
    bb = np.asarray(kz["fp8.B"]).reshape(n, kk)
    c = _f16(kz["fp8.C"]).reshape(m, n)
    nb = -(-kk // 128)
    ref = ofp8.gemm_blockscaled(a, np.ones((m, nb), np.float32), bb,
                                np.ones((-(-n // 128), nb), np.float32))
    err = np.abs(c - ref)
    assert np.all(err <= 1e-3 * np.abs(ref) + 1e-2), err.max()
