"""Attention restatements in float64 (numpy).

- ``attn_fwd`` / ``causal_fwd``: softmax(Q K^T * scale [+ causal mask]) V and the natural-log
  LSE per (batch, head, query) for [B, S, H, D] tensors. The reference's FlashAttention forward
  (perfmodel/testset/gen.py:417-486) computes the same function through an online softmax in
  exp2 form with the log2(e)-folded scale (gen.py:433, :468-472); exp2(x * log2 e) = exp(x),
  so the closed form below is that function without the causal mask's absence.
- ``decode_gqa``: one query per sequence over its own KV rows, query head h reading KV head
  h // (Hq / Hkv) (gen.py:524).
- ``decode_partials`` / ``decode_combine``: the split kernel's per-chunk outputs and the
  combine, one for one with the reference's two kernels;
- ``decode_split``: the same result computed the reference's way, as split-KV partials with
  their log2-unit LSE (gen.py:493-560, LSE at :553) and the exp2-weighted combine
  (gen.py:563-590); used to check that the split form equals the closed form.
"""

from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


def causal_fwd(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
               heads: list[tuple[int, int]] | None = None
               ) -> tuple[np.ndarray, np.ndarray]:
    """O [B, S, H, D] and LSE [B, H, S] in float64; ``heads`` limits the (b, h) pairs
    computed (others are NaN)."""
    return attn_fwd(q, k, v, scale, causal=True, heads=heads)


def attn_fwd(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool,
             heads: list[tuple[int, int]] | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Attention forward over [B, S, H, D] tensors, causal or not (the reference's
    fa_forward is the non-causal one), O and natural-log LSE in float64."""
    bsz, s, h, d = q.shape
    o = np.full((bsz, s, h, d), np.nan)
    lse = np.full((bsz, h, s), np.nan)
    pairs = heads if heads is not None else [(b, hh) for b in range(bsz) for hh in range(h)]
    mask = np.triu(np.ones((s, s), dtype=bool), 1)
    for b, hh in pairs:
        qb = q[b, :, hh, :].astype(np.float64)
        kb = k[b, :, hh, :].astype(np.float64)
        vb = v[b, :, hh, :].astype(np.float64)
        sc = (qb @ kb.T) * scale
        if causal:
            sc[mask] = -np.inf
        mx = sc.max(axis=1, keepdims=True)
        p = np.exp(sc - mx)
        den = p.sum(axis=1, keepdims=True)
        o[b, :, hh, :] = (p @ vb) / den
        lse[b, hh, :] = (mx + np.log(den))[:, 0]
    return o, lse


def decode_gqa(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, seqlens: np.ndarray,
               offsets: np.ndarray, scale: float) -> np.ndarray:
    """O [B, Hq, D] (float64). A sequence of length 0 yields zeros (the kernel's contract)."""
    bsz, hq, d = q.shape
    hkv = kc.shape[1]
    g = hq // hkv
    out = np.zeros((bsz, hq, d))
    for b in range(bsz):
        n, o0 = int(seqlens[b]), int(offsets[b])
        if n <= 0:
            continue
        for h in range(hq):
            kv = h // g
            kb = kc[o0:o0 + n, kv, :].astype(np.float64)
            vb = vc[o0:o0 + n, kv, :].astype(np.float64)
            sc = kb @ q[b, h].astype(np.float64) * scale
            p = np.exp(sc - sc.max())
            out[b, h] = (p @ vb) / p.sum()
    return out


def decode_partials(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, seqlen: int, offset: int,
                    scale: float, chunk: int) -> tuple[np.ndarray, np.ndarray]:
    """The split kernel's outputs for one sequence (gen.py:493-560): per query head and
    KV chunk of ``chunk`` rows the normalised partial o_c [Hq, n_chunks, D] and its log2-unit
    log-sum-exp lse2_c [Hq, n_chunks] = log2(sum_j 2^(s_j scale log2e - m)) + m, m the chunk's
    maximum of s_j scale log2e (gen.py:553)."""
    hq, d = q.shape
    hkv = kc.shape[1]
    grp = hq // hkv
    nch = -(-seqlen // chunk)
    parts = np.zeros((hq, nch, d))
    lse2 = np.zeros((hq, nch))
    for h in range(hq):
        kv = h // grp
        for c in range(nch):
            c0, c1 = c * chunk, min(seqlen, (c + 1) * chunk)
            kb = kc[offset + c0:offset + c1, kv, :].astype(np.float64)
            vb = vc[offset + c0:offset + c1, kv, :].astype(np.float64)
            s2 = kb @ q[h].astype(np.float64) * scale * LOG2E
            m = s2.max()
            p = np.exp2(s2 - m)
            parts[h, c] = (p @ vb) / p.sum()
            lse2[h, c] = np.log2(p.sum()) + m
    return parts, lse2


def decode_combine(parts: np.ndarray, lse2: np.ndarray) -> np.ndarray:
    """The combine kernel (gen.py:563-590): out = sum_c 2^(lse2_c - max) o_c / sum_c
    2^(lse2_c - max), per head; ``parts`` [..., n_chunks, D], ``lse2`` [..., n_chunks]."""
    w = np.exp2(lse2 - lse2.max(axis=-1, keepdims=True))
    return (w[..., None] * parts).sum(-2) / w.sum(-1)[..., None]


def decode_split(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, seqlens: np.ndarray,
                 offsets: np.ndarray, scale: float, chunk: int) -> np.ndarray:
    """The split-KV form: per chunk a normalised partial and lse2 = log2(sum 2^(s*scale*log2e))
    (gen.py:553), then out = sum_c 2^(lse2_c - max) o_c / sum_c 2^(lse2_c - max) (gen.py:579-588).
    """
    bsz, hq, d = q.shape
    hkv = kc.shape[1]
    g = hq // hkv
    out = np.zeros((bsz, hq, d))
    for b in range(bsz):
        n, o0 = int(seqlens[b]), int(offsets[b])
        if n <= 0:
            continue
        for h in range(hq):
            kv = h // g
            parts, lses = [], []
            for c0 in range(0, n, chunk):
                c1 = min(n, c0 + chunk)
                kb = kc[o0 + c0:o0 + c1, kv, :].astype(np.float64)
                vb = vc[o0 + c0:o0 + c1, kv, :].astype(np.float64)
                s2 = kb @ q[b, h].astype(np.float64) * scale * LOG2E
                m = s2.max()
                p = np.exp2(s2 - m)
                parts.append((p @ vb) / p.sum())
                lses.append(np.log2(p.sum()) + m)
            lses_a = np.array(lses)
            w = np.exp2(lses_a - lses_a.max())
            out[b, h] = (w[:, None] * np.array(parts)).sum(0) / w.sum()
    return out
