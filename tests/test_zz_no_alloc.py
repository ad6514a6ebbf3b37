"""rb_fused_attn_hyb_noalloc: the trie attention for callers that cannot
allocate device memory (its scratch is a fixed 16 MiB array owned by the
library). Checked through the C ABI against rb_fused_attn_hyb (caller-provided
scratch) on two calls in a row, at the capacity boundary, and with no rows.
Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest
import torch

from oracle.bf16 import round_bf16
from oracle.inputs import attention_case, chain_seqs, top_up

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _args(q, kp, vp, kn, vn, msk, out, scale):
    from respect_b200 import _lib
    a = _lib.AttnArgs()
    a.dtype = _lib.dtype_code(q.dtype)
    (a.H, a.M, a.D), (a.HK, a.NP, _), a.NN = q.shape, kp.shape, kn.shape[1]
    a.q, (a.sqh, a.sqm, a.sqd) = q.data_ptr(), q.stride()
    a.kp, (a.skph, a.skpn, a.skpd) = kp.data_ptr(), kp.stride()
    a.vp, (a.svph, a.svpn, a.svpd) = vp.data_ptr(), vp.stride()
    a.kn, (a.sknh, a.sknn, a.sknd) = kn.data_ptr(), kn.stride()
    a.vn, (a.svnh, a.svnn, a.svnd) = vn.data_ptr(), vn.stride()
    a.msk, (a.smm, a.smn), a.mask_kind = msk.data_ptr(), msk.stride(), _lib.RB_MASK_BOOL
    a.out, (a.soh, a.som, a.sod) = out.data_ptr(), out.stride()
    a.sm_scale = scale
    return a


def _case(seed, NP, dtype):
    rng = np.random.default_rng(seed)
    seqs = top_up(rng, chain_seqs(rng, 4, 12, 50), 48, 50)
    c = attention_case(seed, H=28, HK=4, NP=NP, seqs=seqs, committed=3)
    conv = (lambda x: round_bf16(x)) if dtype == torch.bfloat16 else (lambda x: x)
    t = {k: torch.from_numpy(np.ascontiguousarray(conv(c[k]))).to(DEV, dtype) for k in ("q", "kp", "vp", "kn", "vn")}
    t["msk"] = torch.from_numpy(c["msk"]).to(DEV)
    return t


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_noalloc_attention_matches_workspace_entry_point(dtype, tol):
    from respect_b200 import _lib
    from respect_b200.kernels.attention import attn_call
    lib = _lib.lib()
    fn = lib.rb_fused_attn_hyb_noalloc
    fn.restype, fn.argtypes = ctypes.c_int, [ctypes.POINTER(_lib.AttnArgs), ctypes.c_void_p]
    stream = torch.cuda.current_stream().cuda_stream
    for seed, NP in ((0, 1536), (1, 700)):          # two calls in a row, different sizes
        t = _case(seed, NP, dtype)
        ref = torch.empty_like(t["q"])
        attn_call(t["q"], t["kp"], t["vp"], t["kn"], t["vn"], t["msk"], ref, 128 ** -0.5)
        out = torch.full_like(t["q"], float("nan"))
        a = _args(t["q"], t["kp"], t["vp"], t["kn"], t["vn"], t["msk"], out, 128 ** -0.5)
        assert fn(ctypes.byref(a), stream) == _lib.RB_OK
        torch.cuda.synchronize()
        assert float((out.float() - ref.float()).abs().max()) <= tol
        assert torch.equal(out, ref)                # same kernels: bitwise equal in fact


def test_noalloc_attention_rejects_oversized_calls():
    from respect_b200 import _lib
    lib = _lib.lib()
    fn = lib.rb_fused_attn_hyb_noalloc
    fn.restype, fn.argtypes = ctypes.c_int, [ctypes.POINTER(_lib.AttnArgs), ctypes.c_void_p]
    t = _case(2, 1536, torch.bfloat16)
    big_q = torch.zeros(28, 1024, 128, device=DEV, dtype=torch.bfloat16)   # 1024 rows: > 16 MiB of partials
    out = torch.empty_like(big_q)
    msk = torch.zeros(1024, t["kn"].shape[1], dtype=torch.bool, device=DEV)
    a = _args(big_q, t["kp"], t["vp"], t["kn"], t["vn"], msk, out, 128 ** -0.5)
    assert fn(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == _lib.RB_ERR_CAPACITY


CAPACITY = 16 << 20     # the library's no-allocation scratch per device


def test_noalloc_attention_capacity_boundary_and_empty_call():
    """The largest fp32 call whose scratch need (rb_fused_attn_hyb_workspace) fits the
    16 MiB array runs and matches the workspace entry point bitwise; one more row
    returns RB_ERR_CAPACITY; a call with no rows does nothing."""
    from respect_b200 import _lib
    from respect_b200.kernels.attention import attn_call
    lib = _lib.lib()
    fn = lib.rb_fused_attn_hyb_noalloc
    fn.restype, fn.argtypes = ctypes.c_int, [ctypes.POINTER(_lib.AttnArgs), ctypes.c_void_p]
    stream = torch.cuda.current_stream().cuda_stream
    H, HK, D, NP, NN = 28, 4, 128, 1536, 32
    need = [lib.rb_fused_attn_hyb_workspace(H, m, D, NP) for m in range(1, 400)]
    fit = max(m for m in range(1, 400) if need[m - 1] <= CAPACITY)
    assert need[fit - 1] <= CAPACITY < need[fit]
    g = torch.Generator(device=DEV).manual_seed(5)
    kp = torch.randn(HK, NP, D, device=DEV, generator=g)
    vp = torch.randn(HK, NP, D, device=DEV, generator=g)
    kn = torch.randn(HK, NN, D, device=DEV, generator=g)
    vn = torch.randn(HK, NN, D, device=DEV, generator=g)
    for M, want in ((fit, _lib.RB_OK), (fit + 1, _lib.RB_ERR_CAPACITY)):
        q = torch.randn(H, M, D, device=DEV, generator=g) / D ** 0.5
        msk = torch.rand(M, NN, device=DEV, generator=g) < 0.5
        msk[:, 0] = True
        out = torch.full_like(q, float("nan"))
        a = _args(q, kp, vp, kn, vn, msk, out, D ** -0.5)
        assert fn(ctypes.byref(a), stream) == want, M
        if want == _lib.RB_OK:
            ref = torch.empty_like(q)
            attn_call(q, kp, vp, kn, vn, msk, ref, D ** -0.5)
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
    a = _args(q, kp, vp, kn, vn, msk, out, D ** -0.5)   # real buffers (torch gives empty views no pointer) ...
    a.M = 0                                             # ... and no rows
    assert fn(ctypes.byref(a), stream) == _lib.RB_OK
