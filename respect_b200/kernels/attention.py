"""Trie-verification attention with a slot-order-independent node sum.

Drop-in for ``respect.kernels.attention.fused_attn_hyb``
(respect/kernels/attention.py:74-96): same argument names, shapes and output.
The tile keyword arguments (BM, BN, num_warps, num_stages) of the Triton
version are accepted and ignored; BNB keeps the reference's divisibility
check on the node count. The computation runs in librespect_b200.so
(rb_fused_attn_hyb): prefix keys in fixed chunks at absolute positions,
nodes one at a time in slot order, fp32 accumulation, one final cast.
"""
from __future__ import annotations

import ctypes

import torch

from respect_b200 import _lib

_MASK_KIND = {torch.bool: _lib.RB_MASK_BOOL, torch.uint8: _lib.RB_MASK_BOOL,
              torch.bfloat16: _lib.RB_MASK_ADD_BF16, torch.float32: _lib.RB_MASK_ADD_F32}


def _unit_inner(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def attn_call(q, kp, vp, kn, vn, msk, out, sm_scale, mask_kind=None, causal_first=0):
    """Launch rb_fused_attn_hyb on explicit (possibly strided) views.

    q, out [H, M, D]; kp, vp [HK, NP, D]; kn, vn [HK, NN, D]; msk [M, NN] (bool,
    or additive bf16/fp32 where 0 means attend) or None with
    mask_kind=RB_MASK_CAUSAL.
    """
    H, M, D = q.shape
    HK, NP, _ = kp.shape
    NN = kn.shape[1]
    a = _lib.AttnArgs()
    a.dtype = _lib.dtype_code(q.dtype)
    a.H, a.M, a.D, a.HK, a.NP, a.NN = H, M, D, HK, NP, NN
    a.q, (a.sqh, a.sqm, a.sqd) = q.data_ptr(), q.stride()
    a.kp, (a.skph, a.skpn, a.skpd) = kp.data_ptr(), kp.stride()
    a.vp, (a.svph, a.svpn, a.svpd) = vp.data_ptr(), vp.stride()
    a.kn, (a.sknh, a.sknn, a.sknd) = kn.data_ptr(), kn.stride()
    a.vn, (a.svnh, a.svnn, a.svnd) = vn.data_ptr(), vn.stride()
    if msk is None:
        a.msk, a.mask_kind, a.smm, a.smn = None, _lib.RB_MASK_CAUSAL, 0, 0
    else:
        a.msk, (a.smm, a.smn) = msk.data_ptr(), msk.stride()
        a.mask_kind = _MASK_KIND[msk.dtype] if mask_kind is None else mask_kind
    a.causal_first = int(causal_first)
    a.out, (a.soh, a.som, a.sod) = out.data_ptr(), out.stride()
    a.sm_scale = float(sm_scale)
    nbytes = _lib.lib().rb_fused_attn_hyb_workspace(H, M, D, NP)
    ws = _lib.workspace(q, nbytes)
    _lib.call("rb_fused_attn_hyb", ctypes.byref(a), ws.data_ptr() if ws is not None else None,
              nbytes, _lib.stream_of(q))
    return out


def fused_attn_hyb(q, kp, vp, kn, vn, msk, sm_scale=None,
                   BM=64, BN=128, BNB=16, num_warps=4, num_stages=1):
    """q [H, M, D], kp/vp [HK, NP, D], kn/vn [HK, NN, D], msk [M, NN] bool -> [H, M, D]."""
    H, M, D = q.shape
    NN = kn.shape[1]
    assert NN % BNB == 0  # same precondition as the reference (attention.py:79)
    if sm_scale is None:
        sm_scale = D ** -0.5
    q, kp, vp, kn, vn = (_unit_inner(t) for t in (q, kp, vp, kn, vn))
    out = torch.empty_like(q)
    return attn_call(q, kp, vp, kn, vn, msk, out, sm_scale)
