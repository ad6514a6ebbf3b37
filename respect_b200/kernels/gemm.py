"""Linear layer whose result does not depend on the number of rows.

Drop-in for ``respect.kernels.gemm.linear`` (respect/kernels/gemm.py:30-41).
The tile keyword arguments are accepted and ignored: the native kernel
(rb_linear, tcgen05 + TMA) fixes its own tile and K split from (N, K) alone,
so a row gives the same bits alone or with other rows.
"""
from __future__ import annotations

import torch

from respect_b200 import _lib


def linear(x, w, BM=32, BN=128, BK=64, num_warps=4, num_stages=2, out_dtype=None):
    """x (..., K) @ w (N, K)^T -> (..., N). Bias is handled by the caller."""
    K = x.shape[-1]
    xs = x.reshape(-1, K).contiguous()
    M = xs.shape[0]
    N = w.shape[0]
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError("respect_b200.linear takes bf16 x and w")
    if w.stride(-1) != 1:
        w = w.contiguous()
    od = out_dtype or x.dtype
    out = torch.empty((M, N), device=x.device, dtype=od)
    nbytes = _lib.lib().rb_linear_workspace(M, N, K)
    ws = _lib.workspace(xs, nbytes)
    _lib.call("rb_linear", xs.data_ptr(), xs.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
              out.stride(0), _lib.dtype_code(od), M, N, K,
              ws.data_ptr() if ws is not None else None, nbytes, _lib.stream_of(xs))
    return out.reshape(*x.shape[:-1], N)


def pack_weight(w: torch.Tensor, bn: int = 0) -> torch.Tensor:
    """Copy of w [N, K] (bf16) in the packed tile layout the weight-streaming
    kernel reads contiguously: [ceil(N/BN)][ceil(K/64)][BN][64], zero padded.
    bn=0 uses the tile width linear() picks for (N, K)."""
    N, K = w.shape
    if w.stride(-1) != 1:
        w = w.contiguous()
    nbytes = _lib.lib().rb_linear_packed_bytes(N, K, bn)
    out = torch.empty(nbytes // 2, dtype=torch.bfloat16, device=w.device)
    _lib.call("rb_pack_linear_weight", w.data_ptr(), w.stride(0), N, K, bn, out.data_ptr(), _lib.stream_of(w))
    return out


def linear_packed(x, w_packed, N, out_dtype=None):
    """linear(x, w) for a weight packed by pack_weight(w) (bn=0): bitwise equal results."""
    K = x.shape[-1]
    xs = x.reshape(-1, K).contiguous()
    M = xs.shape[0]
    od = out_dtype or x.dtype
    out = torch.empty((M, N), device=x.device, dtype=od)
    nbytes = _lib.lib().rb_linear_workspace(M, N, K)
    ws = _lib.workspace(xs, nbytes)
    _lib.call("rb_linear_packed", xs.data_ptr(), xs.stride(0), w_packed.data_ptr(), out.data_ptr(), out.stride(0),
              _lib.dtype_code(od), M, N, K, ws.data_ptr() if ws is not None else None, nbytes, _lib.stream_of(xs))
    return out.reshape(*x.shape[:-1], N)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Gate and up weights [F, K] -> [2F, K] in alternating 128-row blocks (gate, up, gate, ...)."""
    f, k = gate.shape
    if f % 128 != 0 or up.shape != gate.shape:
        raise ValueError("gate/up weights must share a shape with a multiple of 128 rows")
    return torch.stack([gate.reshape(f // 128, 128, k), up.reshape(f // 128, 128, k)], dim=1).reshape(2 * f, k)


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """The packed weight linear_swiglu_packed reads (interleaved, then packed with BN = 256)."""
    return pack_weight(interleave_gate_up(gate, up), bn=256)


def linear_swiglu_packed(x, w_gu_packed, F):
    """silu(x @ gate^T) * (x @ up^T) -> (..., F) bf16 in one launch (rb_linear_swiglu_packed);
    bitwise equal to silu_mul(linear(x, gate), linear(x, up)) computed on the interleaved weight."""
    K = x.shape[-1]
    xs = x.reshape(-1, K).contiguous()
    if xs.dtype != torch.bfloat16 or w_gu_packed.dtype != torch.bfloat16:
        raise TypeError("respect_b200.linear_swiglu_packed takes bf16 x and weights")
    M = xs.shape[0]
    out = torch.empty((M, F), device=x.device, dtype=torch.bfloat16)
    _lib.call("rb_linear_swiglu_packed", xs.data_ptr(), xs.stride(0), w_gu_packed.data_ptr(), out.data_ptr(),
              out.stride(0), M, F, K, _lib.stream_of(xs))
    return out.reshape(*x.shape[:-1], F)
