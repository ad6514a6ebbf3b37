"""Linear, RMSNorm, RoPE and SiLU*mul, restated in numpy with the reference's
rounding points.

* `linear`    respect/kernels/gemm.py:11-27 — x @ w^T with fp32 accumulation,
              output in the input dtype or fp32 (lm_head, patch.py:23, 33-34).
* `rmsnorm`   respect/kernels/rmsnorm.py:12-22 — upcast, mean of squares,
              rsqrt, downcast to the input dtype, times weight, downcast.
* `rope`      respect/system/fused.py:45-64 — x*cos + rotate_half(x)*sin, each
              product and the sum rounded to bf16 for bf16 output.
* `silu_mul`  respect/system/fused.py:106-113 — bf16(bf16(g/(1+exp(-g))) * u).
* `rope_cos_sin` — the text rotary table of HF Qwen3-VL with all three mRoPE
              axes equal (respect/decoding/verify.py:31-33 sets them equal):
              inv_freq = 1/theta^(2i/D), freqs = pos*inv_freq, emb = [f, f].
"""
from __future__ import annotations

import numpy as np

from oracle.bf16 import round_bf16


def linear(x, w, out_bf16=True):
    y = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
    return round_bf16(y) if out_bf16 else y.astype(np.float32)


def rmsnorm(x, w, eps, bf16=True):
    x = np.asarray(x, np.float32)
    var = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    xh = x * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))
    if bf16:
        xh = round_bf16(xh)
    y = np.asarray(w, np.float32) * xh
    return round_bf16(y) if bf16 else y


def rotate_half(x):
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def rope(x, cos, sin, bf16=True):
    """x [..., L, D]; cos/sin broadcastable to x."""
    x = np.asarray(x, np.float32)
    a = x * np.asarray(cos, np.float32)
    r = rotate_half(x) * np.asarray(sin, np.float32)
    if bf16:
        a, r = round_bf16(a), round_bf16(r)
    y = a + r
    return round_bf16(y) if bf16 else y


def silu_mul(g, u, bf16=True):
    g = np.asarray(g, np.float32)
    u = np.asarray(u, np.float32)
    with np.errstate(over="ignore"):
        s = g / (np.float32(1.0) + np.exp(-g))
    if bf16:
        return round_bf16(round_bf16(s) * u)
    return (s * u).astype(np.float32)


def rope_inv_freq(head_dim, theta):
    exps = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / (np.float32(theta) ** exps)).astype(np.float32)


def rope_cos_sin(positions, head_dim, theta, bf16=True):
    inv = rope_inv_freq(head_dim, theta)
    f = np.asarray(positions, np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([f, f], axis=-1)
    c, s = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    return (round_bf16(c), round_bf16(s)) if bf16 else (c, s)
