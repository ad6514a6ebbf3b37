"""Output-preserving RoPE and SwiGLU kernels.

Drop-ins for ``respect.system.fused.rope`` and ``silu_mul``
(respect/system/fused.py:67-75, 116-123): every elementwise operation is
rounded where PyTorch eager rounds it (bf16 after each op for bf16 data, fp32
otherwise, no FMA contraction), so results are bitwise equal to the eager
``q*cos + rotate_half(q)*sin`` and ``silu(g) * u``.
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
