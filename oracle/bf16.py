"""bf16 rounding in numpy (round-to-nearest-even on the fp32 bit pattern).

Restates the rounding the reference relies on at every bf16 cast
(respect/system/fused.py:32-42 states the same rule for its kernels).
"""
from __future__ import annotations

import numpy as np


def round_bf16(x) -> np.ndarray:
    """fp32 -> nearest bf16 value (ties to even), returned as fp32. NaN stays NaN."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).reshape(a.shape)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def bf16_bits(x) -> np.ndarray:
    """fp32 values (already bf16-representable after rounding) -> uint16 bit patterns."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
