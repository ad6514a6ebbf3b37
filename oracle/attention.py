"""Trie-verification attention, restated in numpy fp32.

`fused_attn_hyb` follows respect/kernels/attention.py:24-71 step by step: the
prefix [0, NP) in BN-key tiles with an online softmax (:36-50; probabilities
cast to the value dtype for the P.V product, :48), then the node slots in
blocks of BNB whose scores are masked to -inf (:52-58) and folded in one slot
at a time in slot order (:59-67), then one divide (:69).
`sdpa` is the reference's eager path: plain masked softmax attention over
[prefix | nodes] (what HF SDPA computes when dispatch falls back,
respect/kernels/dispatch.py:113, 160-171).
"""
from __future__ import annotations

import numpy as np

from oracle.bf16 import round_bf16


def fused_attn_hyb(q, kp, vp, kn, vn, msk, sm_scale=None, BN=128, BNB=16, p_bf16=False):
    q = np.asarray(q, np.float32)
    kp, vp, kn, vn = (np.asarray(t, np.float32) for t in (kp, vp, kn, vn))
    msk = np.asarray(msk, bool)
    H, M, D = q.shape
    HK, NP, _ = kp.shape
    NN = kn.shape[1]
    G = H // HK
    scale = np.float32(D ** -0.5 if sm_scale is None else sm_scale)
    out = np.empty((H, M, D), np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        for h in range(H):
            kv = h // G
            qh = q[h]
            m = np.full(M, -np.inf, np.float32)
            l = np.zeros(M, np.float32)
            acc = np.zeros((M, D), np.float32)
            for s0 in range(0, NP, BN):
                k = kp[kv, s0:s0 + BN]
                v = vp[kv, s0:s0 + BN]
                s = (qh @ k.T) * scale
                m_new = np.maximum(m, s.max(axis=1))
                alpha = np.exp(m - m_new)
                p = np.exp(s - m_new[:, None])
                pv = round_bf16(p) if p_bf16 else p
                acc = acc * alpha[:, None] + pv @ v
                l = l * alpha + p.sum(axis=1)
                m = m_new
            for s0 in range(0, NN, BNB):
                k = kn[kv, s0:s0 + BNB]
                s = (qh @ k.T) * scale
                s = np.where(msk[:, s0:s0 + BNB], s, np.float32(-np.inf))
                for j in range(s.shape[1]):
                    sj = s[:, j]
                    m_new = np.maximum(m, sj)
                    alpha = np.exp(m - m_new)
                    p = np.exp(sj - m_new)
                    acc = acc * alpha[:, None] + p[:, None] * vn[kv, s0 + j][None, :]
                    l = l * alpha + p
                    m = m_new
            out[h] = acc / l[:, None]
    return out


def sdpa(q, kp, vp, kn, vn, msk, sm_scale=None):
    """Masked softmax attention in float64: keys = prefix (always open) + allowed nodes."""
    q = np.asarray(q, np.float64)
    H, M, D = q.shape
    HK = kp.shape[0]
    G = H // HK
    scale = D ** -0.5 if sm_scale is None else sm_scale
    k = np.concatenate([np.asarray(kp, np.float64), np.asarray(kn, np.float64)], axis=1)
    v = np.concatenate([np.asarray(vp, np.float64), np.asarray(vn, np.float64)], axis=1)
    allow = np.concatenate([np.ones((M, kp.shape[1]), bool), np.asarray(msk, bool)], axis=1)
    out = np.empty((H, M, D), np.float64)
    for h in range(H):
        s = (q[h] @ k[h // G].T) * scale
        s = np.where(allow, s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[h] = p @ v[h // G]
    return out
