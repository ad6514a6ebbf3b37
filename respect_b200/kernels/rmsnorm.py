"""RMS normalization whose result does not depend on the number of rows.

Drop-in for ``respect.kernels.rmsnorm.rmsnorm`` (respect/kernels/rmsnorm.py:25-32):
one row per thread group, fixed-order sum, PyTorch's rounding points
(upcast, mean of squares, rsqrt, downcast, times weight). Runs rb_rmsnorm.
"""
from __future__ import annotations

import torch

from respect_b200 import _lib


def rmsnorm(x, w, eps):
    xs = x.reshape(-1, x.shape[-1]).contiguous()
    M, N = xs.shape
    out = torch.empty_like(xs)
    w = w.contiguous()
    _lib.call("rb_rmsnorm", xs.data_ptr(), w.data_ptr(), out.data_ptr(), M, N, float(eps),
              _lib.dtype_code(xs.dtype), _lib.dtype_code(w.dtype), _lib.stream_of(xs))
    return out.reshape(x.shape)
