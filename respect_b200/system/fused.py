"""Output-preserving elementwise kernels.

Drop-ins for ``respect.system.fused`` (respect/system/fused.py:67-194): `rope`,
`silu_mul`, and the Prefill norm pieces `add_sq`, `norm_from` and `rmsnorm`.
Every elementwise operation is rounded where PyTorch eager rounds it (bf16
after each op for bf16 data, fp32 otherwise, no FMA contraction), so results
are bitwise equal to the eager ``q*cos + rotate_half(q)*sin``, ``silu(g) * u``,
``r + h`` and HF's RMSNorm (whose row mean PyTorch computes itself).
"""
from __future__ import annotations

import torch

from respect_b200 import _lib


def rope(x, cos, sin):
    """q*cos + rotate_half(q)*sin. x [B, H, L, D], cos/sin [B, L, D]."""
    out_dtype = torch.promote_types(x.dtype, cos.dtype)
    B, H, L, D = x.shape
    y = torch.empty((B, H, L, D), device=x.device, dtype=out_dtype)
    cos, sin = cos.contiguous(), sin.contiguous()
    if cos.shape != (B, L, D) and cos.dim() == 3 and cos.shape[0] == 1:
        cos, sin = cos.expand(B, L, D), sin.expand(B, L, D)
    _lib.call("rb_rope", x.data_ptr(), *x.stride(), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
              cos.stride(1), y.data_ptr(), B, H, L, D, _lib.dtype_code(x.dtype),
              _lib.dtype_code(cos.dtype), _lib.dtype_code(out_dtype), _lib.stream_of(x))
    return y


def silu_mul(g, u):
    """silu(g) * u with eager rounding points (bf16 or fp32, matching dtypes)."""
    if g.dtype != u.dtype or g.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("silu_mul takes two bf16 or two fp32 tensors")
    g, u = g.contiguous(), u.contiguous()
    y = torch.empty_like(g)
    _lib.call("rb_silu_mul", g.data_ptr(), u.data_ptr(), y.data_ptr(), g.numel(),
              _lib.dtype_code(g.dtype), _lib.stream_of(g))
    return y


def add_sq(r, h):
    """x = r + h with PyTorch type promotion and rounding, and x.float() ** 2 (fused.py:184-194)."""
    out_dtype = torch.promote_types(r.dtype, h.dtype)
    rs, hs = r.reshape(-1, r.shape[-1]).contiguous(), h.reshape(-1, h.shape[-1]).contiguous()
    x = torch.empty(rs.shape, device=r.device, dtype=out_dtype)
    sq = torch.empty(rs.shape, device=r.device, dtype=torch.float32)
    _lib.call("rb_add_sq", rs.data_ptr(), hs.data_ptr(), x.data_ptr(), sq.data_ptr(), rs.numel(),
              _lib.dtype_code(rs.dtype), _lib.dtype_code(hs.dtype), _lib.dtype_code(out_dtype), _lib.stream_of(rs))
    return x, sq


def norm_from(xs, sq, w, eps):
    """HF RMSNorm of xs [M, N] given sq = xs.float() ** 2: the mean by PyTorch, the rest here (fused.py:160-168)."""
    M, N = xs.shape
    var = sq.mean(-1).contiguous()
    out_dtype = torch.promote_types(w.dtype, xs.dtype)
    y = torch.empty((M, N), device=xs.device, dtype=out_dtype)
    xs, w = xs.contiguous(), w.contiguous()
    _lib.call("rb_norm_apply", xs.data_ptr(), var.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, float(eps),
              _lib.dtype_code(xs.dtype), _lib.dtype_code(w.dtype), _lib.dtype_code(out_dtype), _lib.stream_of(xs))
    return y


def rmsnorm(x, w, eps):
    """HF RMSNorm, bit for bit with eager (fused.py:171-177); the deterministic, row-count-invariant
    norm of the verify path is respect_b200.kernels.rmsnorm."""
    xs = x.reshape(-1, x.shape[-1]).contiguous()
    sq = torch.empty(xs.shape, device=x.device, dtype=torch.float32)
    _lib.call("rb_add_sq", xs.data_ptr(), None, None, sq.data_ptr(), xs.numel(), _lib.dtype_code(xs.dtype),
              _lib.RB_F32, _lib.RB_F32, _lib.stream_of(xs))
    return norm_from(xs, sq, w, eps).reshape(x.shape)
