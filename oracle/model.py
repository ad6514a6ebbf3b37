"""One verify forward of a Qwen3-style decoder, restated in numpy.

Follows what respect/decoding/verify.py:12-46 runs: node i of the trie gets
KV slot prompt_len+base+i and rotary position prompt_len+base+depth(i)
(:24-33), and attends to the prefix, the committed tokens and its own trie
ancestors (:35-41). The layer body is HF's Qwen3VLTextDecoderLayer (q_norm /
k_norm on the head dim, RoPE, attention, o_proj, residual, post-attention
norm, SwiGLU MLP, residual) with the dedicated kernels of
respect/kernels/patch.py:70-107 (linear: fp32 accumulation, bf16 out; lm_head
fp32 out), rounding to bf16 where the bf16 eager path rounds
(`bf16=True`), or in fp32 throughout (`bf16=False`).

Weights are a dict of numpy fp32 arrays:
  embed [V, h], lm_head [V, h], final_norm [h], layers: list of dicts with
  wq [H*D, h], wk [HK*D, h], wv [HK*D, h], wo [h, H*D], wg [F, h], wu [F, h],
  wd [h, F], in_norm [h], post_norm [h], q_norm [D], k_norm [D].
KV: per layer k[l], v[l] arrays [HK, S, D] (updated in place).
"""
from __future__ import annotations

import numpy as np

from oracle import attention as oatt
from oracle import ops
from oracle.bf16 import round_bf16
from oracle.trie import ancestry


def _r(x, bf16):
    return round_bf16(x) if bf16 else np.asarray(x, np.float32)


def verify_step(W, cfg, ids, parents, depths, prompt_len, base, kc, vc, bf16=True, layers=None,
                return_hidden=False):
    """Returns fp32 logits [q, V] (and the final residual stream if asked)."""
    H, HK, D = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    eps, theta = cfg["rms_eps"], cfg["rope_theta"]
    q = len(ids)
    start = prompt_len + base
    slots = np.arange(start, start + q)
    pos = start + np.asarray(depths)
    cos, sin = ops.rope_cos_sin(pos, D, theta, bf16=bf16)
    anc = ancestry(list(parents))
    n_node = base + q
    msk = np.zeros((q, n_node), bool)
    msk[:, :base] = True
    msk[:, base:] = anc
    h = _r(W["embed"][np.asarray(ids)], bf16)
    L = W["layers"] if layers is None else W["layers"][:layers]
    for li, lw in enumerate(L):
        x = ops.rmsnorm(h, lw["in_norm"], eps, bf16)
        qh = ops.linear(x, lw["wq"], bf16).reshape(q, H, D)
        kh = ops.linear(x, lw["wk"], bf16).reshape(q, HK, D)
        vh = ops.linear(x, lw["wv"], bf16).reshape(q, HK, D)
        qh = ops.rmsnorm(qh, lw["q_norm"], eps, bf16)
        kh = ops.rmsnorm(kh, lw["k_norm"], eps, bf16)
        qh = ops.rope(qh.transpose(1, 0, 2), cos[None], sin[None], bf16)      # [H, q, D]
        kh = ops.rope(kh.transpose(1, 0, 2), cos[None], sin[None], bf16)      # [HK, q, D]
        kc[li][:, slots] = kh
        vc[li][:, slots] = vh.transpose(1, 0, 2)
        kp, vp = kc[li][:, :prompt_len], vc[li][:, :prompt_len]
        kn, vn = kc[li][:, prompt_len:prompt_len + n_node], vc[li][:, prompt_len:prompt_len + n_node]
        a = oatt.fused_attn_hyb(qh, kp, vp, kn, vn, msk, D ** -0.5, p_bf16=bf16)  # [H, q, D]
        a = _r(a, bf16).transpose(1, 0, 2).reshape(q, H * D)
        h = _r(h + ops.linear(a, lw["wo"], bf16), bf16)
        x = ops.rmsnorm(h, lw["post_norm"], eps, bf16)
        g = ops.linear(x, lw["wg"], bf16)
        u = ops.linear(x, lw["wu"], bf16)
        act = ops.silu_mul(g, u, bf16)
        h = _r(h + ops.linear(act, lw["wd"], bf16), bf16)
    x = ops.rmsnorm(h, W["final_norm"], eps, bf16)
    logits = ops.linear(x, W["lm_head"], out_bf16=False)
    return (logits, h) if return_hidden else logits


def prefill(W, cfg, tokens, kc, vc, chunk=64, bf16=True):
    """Prompt KV by chained steps: chunk c is a chain whose prompt is the c * chunk
    tokens before it (prompt_len c * chunk, base 0)."""
    toks = np.asarray(tokens)
    for s in range(0, len(toks), chunk):
        part = toks[s:s + chunk]
        n = len(part)
        verify_step(W, cfg, part, np.arange(-1, n - 1), np.arange(n), s, 0, kc, vc, bf16=bf16)


def weights_from_engine(w, cfg):
    """numpy fp32 copies of respect_b200 DecoderWeights (torch bf16 on a device)."""
    import torch

    def f(t):
        return t.detach().float().cpu().numpy()

    H, HK, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    layers = []
    for lw in w.layers:
        qkv = f(lw["wqkv"])
        f2, hdim = lw["wgu"].shape
        gu = lw["wgu"].view(f2 // 256, 2, 128, hdim)
        layers.append(dict(
            wq=qkv[:H * D], wk=qkv[H * D:(H + HK) * D], wv=qkv[(H + HK) * D:],
            wo=f(lw["wo"]), wg=f(gu[:, 0].reshape(f2 // 2, hdim)), wu=f(gu[:, 1].reshape(f2 // 2, hdim)),
            wd=f(lw["wd"]), in_norm=f(lw["in_norm"]), post_norm=f(lw["post_norm"]),
            q_norm=f(lw["q_norm"]), k_norm=f(lw["k_norm"])))
    del torch
    return dict(embed=f(w.embed), lm_head=f(w.lm_head), final_norm=f(w.final_norm), layers=layers)


def cfg_dict(cfg):
    return dict(n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim,
                rms_eps=cfg.rms_eps, rope_theta=cfg.rope_theta)
