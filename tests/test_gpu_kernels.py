"""Parity of the native kernels (through the C ABI) with the oracle, the
reference's golden outputs and PyTorch eager (the bit-exactness target of
RoPE / SiLU*mul). Tolerances: fp32 attention 1e-5 max-abs, bf16 2e-2 max-abs
(BASELINE north star); integer and mask outputs bit-exact."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import ops as oops
from oracle import trie as otrie
from oracle.bf16 import from_bf16_bits, round_bf16
from oracle.inputs import attention_case, chain_seqs, checksum, top_up

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def pad_rows(c, MP=None):
    """Dispatch layout: rows padded to 64, padding rows open node 0 (dispatch.py:94-115)."""
    M = c["q"].shape[1]
    MP = MP or ((M + 63) // 64) * 64
    q = np.zeros((c["q"].shape[0], MP, c["q"].shape[2]), np.float32)
    q[:, :M] = c["q"]
    msk = np.zeros((MP, c["msk"].shape[1]), bool)
    msk[:M] = c["msk"]
    msk[M:, 0] = True
    return q, msk


# ---------------------------------------------------------------- attention
def test_attention_config1_fp32_matches_reference():
    from respect_b200.kernels.attention import fused_attn_hyb
    kern = np.load(G / "kernels.npz")
    c = attention_case(0)
    assert checksum(*[c[k] for k in ("q", "kp", "vp", "kn", "vn", "msk")]) == str(kern["attn_c1_checksum"])
    q, msk = pad_rows(c)
    out = fused_attn_hyb(T(q), T(c["kp"]), T(c["vp"]), T(c["kn"]), T(c["vn"]), T(msk, torch.bool))
    got = out[:, :48].cpu().numpy()
    assert np.abs(got - kern["attn_c1_out"]).max() < 1e-5          # reference kernel (Triton, interpreted)
    eager = oatt.sdpa(c["q"], c["kp"], c["vp"], c["kn"], c["vn"], c["msk"])
    assert np.abs(got - eager).max() < 1e-5                         # reference eager path


@pytest.mark.parametrize("NP,committed", [(3000, 0), (3000, 37), (700, 5), (0, 3), (1, 0), (512, 0), (513, 2)])
def test_attention_bf16_vs_oracle(NP, committed):
    from respect_b200.kernels.attention import fused_attn_hyb
    rng = np.random.default_rng(NP + committed)
    seqs = top_up(rng, chain_seqs(rng, 4, 32, 50), 128, 50)
    c = attention_case(7, H=28, HK=4, NP=NP, seqs=seqs, committed=committed)
    b = {k: round_bf16(c[k]) for k in ("q", "kp", "vp", "kn", "vn")}
    q, msk = pad_rows(dict(q=b["q"], msk=c["msk"]))
    out = fused_attn_hyb(T(q, torch.bfloat16), T(b["kp"], torch.bfloat16), T(b["vp"], torch.bfloat16),
                         T(b["kn"], torch.bfloat16), T(b["vn"], torch.bfloat16), T(msk, torch.bool))
    got = out[:, :q.shape[1]].float().cpu().numpy()[:, :c["q"].shape[1]]
    ref = oatt.fused_attn_hyb(b["q"], b["kp"], b["vp"], b["kn"], b["vn"], c["msk"], p_bf16=True)
    assert np.abs(got - ref).max() < 2e-2
    eager = oatt.sdpa(b["q"], b["kp"], b["vp"], b["kn"], b["vn"], c["msk"])
    assert np.abs(got - eager).max() < 2e-2


@pytest.mark.parametrize("NP,committed", [(1, 0), (31, 2), (33, 0), (700, 5), (3000, 37)])
def test_attention_fp32_vs_oracle_and_row_invariance(NP, committed):
    """fp32 path (three tf32 products per term) at prefix lengths that leave partial
    32-key tiles and key groups without keys: within 1e-5 of the oracle and of
    eager, and every row alone bitwise equal to its row of the full call."""
    from respect_b200.kernels.attention import attn_call, fused_attn_hyb
    rng = np.random.default_rng(NP + 11 * committed)
    seqs = top_up(rng, chain_seqs(rng, 4, 32, 50), 128, 50)
    c = attention_case(5, H=28, HK=4, NP=NP, seqs=seqs, committed=committed)
    q, msk = pad_rows(c)
    out = fused_attn_hyb(T(q), T(c["kp"]), T(c["vp"]), T(c["kn"]), T(c["vn"]), T(msk, torch.bool))
    M = c["q"].shape[1]
    got = out[:, :M].cpu().numpy()
    ref = oatt.fused_attn_hyb(c["q"], c["kp"], c["vp"], c["kn"], c["vn"], c["msk"])
    assert np.abs(got - ref).max() < 1e-5
    eager = oatt.sdpa(c["q"], c["kp"], c["vp"], c["kn"], c["vn"], c["msk"])
    assert np.abs(got - eager).max() < 1e-5
    full = torch.empty(28, M, 128, device=DEV)
    t = {k: T(c[k]) for k in ("q", "kp", "vp", "kn", "vn")}
    mt = T(c["msk"], torch.bool)
    attn_call(t["q"], t["kp"], t["vp"], t["kn"], t["vn"], mt, full, 128 ** -0.5)
    for r in (0, 15, 16, M - 1):
        o1 = torch.empty(28, 1, 128, device=DEV)
        attn_call(t["q"][:, r:r + 1], t["kp"], t["vp"], t["kn"], t["vn"], mt[r:r + 1], o1, 128 ** -0.5)
        assert torch.equal(o1[:, 0], full[:, r])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_slot_layout_invariance(dtype):
    """The reference's own check (tests/test_kernel_invariance.py:30-54): the same 26
    node values in slots 0-25 vs 0-17 + 200-207 give bitwise equal outputs."""
    from respect_b200.kernels.attention import fused_attn_hyb
    g = torch.Generator(device=DEV).manual_seed(0)
    H, HK, D, NP, n = 32, 8, 128, 300, 26
    q = torch.randn(H, 64, D, device=DEV, generator=g).to(dtype)
    kp = torch.randn(HK, NP, D, device=DEV, generator=g).to(dtype)
    vp = torch.randn(HK, NP, D, device=DEV, generator=g).to(dtype)
    kv_k = torch.randn(HK, n, D, device=DEV, generator=g).to(dtype)
    kv_v = torch.randn(HK, n, D, device=DEV, generator=g).to(dtype)
    NN = 224
    outs = []
    for slots in (list(range(n)), list(range(18)) + list(range(200, 208))):
        kn = torch.zeros(HK, NN, D, device=DEV, dtype=dtype)
        vn = torch.zeros_like(kn)
        msk = torch.zeros(64, NN, device=DEV, dtype=torch.bool)
        for j, s in enumerate(slots):
            kn[:, s] = kv_k[:, j]
            vn[:, s] = kv_v[:, j]
        msk[:, slots] = True
        outs.append(fused_attn_hyb(q, kp, vp, kn, vn, msk, BM=64, BN=128, BNB=16))
    assert torch.equal(outs[0], outs[1])


# The reference's layout sweep (scripts/run_kernel_order.py:32-125): the same 26
# node keys / values placed consecutively, at 0-17 + 200-207, and at 5 seeded
# random sorted slot sets inside NPAD = 256 node slots; one query row attends
# them (padding rows open slot 0).
LAYOUT_NPAD, LAYOUT_N = 256, 26


def _layouts():
    import random
    r = random.Random(0)
    out = [list(range(LAYOUT_N)), list(range(18)) + list(range(200, 200 + LAYOUT_N - 18))]
    out += [sorted(r.sample(range(LAYOUT_NPAD), LAYOUT_N)) for _ in range(5)]
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_layout_sweep(dtype):
    """Consecutive, scattered and 5 random layouts at NPAD=256 give bitwise equal
    outputs (28 / 4 heads, a 3,000-key prefix, as in the config-3 step)."""
    from respect_b200.kernels.attention import fused_attn_hyb
    g = torch.Generator(device=DEV).manual_seed(11)
    H, HK, D, NP = 28, 4, 128, 3000
    q1 = (torch.randn(H, 1, D, device=DEV, generator=g) / D ** 0.5).to(dtype)
    kp = torch.randn(HK, NP, D, device=DEV, generator=g).to(dtype)
    vp = torch.randn(HK, NP, D, device=DEV, generator=g).to(dtype)
    K = torch.randn(HK, LAYOUT_N, D, device=DEV, generator=g).to(dtype)
    V = torch.randn(HK, LAYOUT_N, D, device=DEV, generator=g).to(dtype)
    outs = []
    for slots in _layouts():
        kn = torch.zeros(HK, LAYOUT_NPAD, D, device=DEV, dtype=dtype)
        vn = torch.zeros_like(kn)
        msk = torch.zeros(64, LAYOUT_NPAD, device=DEV, dtype=torch.bool)
        for i, c in enumerate(slots):
            kn[:, c] = K[:, i]
            vn[:, c] = V[:, i]
            msk[0, c] = True
        msk[1:, 0] = True
        q = torch.zeros(H, 64, D, device=DEV, dtype=dtype)
        q[:, 0] = q1[:, 0]
        outs.append(fused_attn_hyb(q, kp, vp, kn, vn, msk)[:, 0].clone())
    for o in outs[1:]:
        assert torch.equal(outs[0], o)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attention_row_count_and_mask_kind_invariance(dtype):
    from respect_b200.kernels.attention import attn_call
    from respect_b200 import _lib
    rng = np.random.default_rng(1)
    seqs = top_up(rng, chain_seqs(rng, 4, 32, 50), 128, 50)
    c = attention_case(3, NP=3000, seqs=seqs, committed=9)
    b = {k: T(round_bf16(c[k]), dtype) for k in ("q", "kp", "vp", "kn", "vn")}
    msk = T(c["msk"], torch.bool)
    full = torch.empty_like(b["q"])
    attn_call(b["q"], b["kp"], b["vp"], b["kn"], b["vn"], msk, full, 128 ** -0.5)
    # additive mask in the data's dtype (dispatch passes allow = mask == 0)
    add = torch.where(msk, 0.0, torch.finfo(dtype).min).to(dtype)
    o2 = torch.empty_like(full)
    attn_call(b["q"], b["kp"], b["vp"], b["kn"], b["vn"], add, o2, 128 ** -0.5)
    assert torch.equal(full, o2)
    # every row alone (M = 1) equals its row of the full call
    for r in (0, 1, 63, 64, 100, 127):
        o1 = torch.empty(28, 1, 128, device=DEV, dtype=dtype)
        attn_call(b["q"][:, r:r + 1], b["kp"], b["vp"], b["kn"], b["vn"], msk[r:r + 1], o1, 128 ** -0.5)
        assert torch.equal(o1[:, 0], full[:, r])
    # causal mode equals the explicit causal bool mask
    NN = b["kn"].shape[1]
    first = NN - 16 - 3
    cm = (torch.arange(NN, device=DEV)[None, :] <= torch.arange(16, device=DEV)[:, None] + first)
    o3 = torch.empty(28, 16, 128, device=DEV, dtype=dtype)
    o4 = torch.empty_like(o3)
    attn_call(b["q"][:, :16], b["kp"], b["vp"], b["kn"], b["vn"], cm, o3, 128 ** -0.5)
    attn_call(b["q"][:, :16], b["kp"], b["vp"], b["kn"], b["vn"], None, o4, 128 ** -0.5,
              mask_kind=_lib.RB_MASK_CAUSAL, causal_first=first)
    assert torch.equal(o3, o4)


# ---------------------------------------------------------------- linear
def _bf16_close(got, ref, K):
    """bf16 output vs an fp64 reference: within one bf16 ulp of the magnitude plus
    the fp32-order noise of a K-long sum."""
    tol = np.abs(ref) * 2 ** -7 + 1e-6 * np.sqrt(K) * np.abs(ref).max()
    return np.all(np.abs(got - ref) <= tol)


@pytest.mark.parametrize("M,N,K,out", [(64, 1024, 4096, "bf16"), (128, 4608, 3584, "bf16"),
                                       (128, 3584, 18944, "bf16"), (1, 37888, 3584, "bf16"),
                                       (300, 1000, 200, "bf16"), (129, 152064, 512, "f32"),
                                       (7, 208 * 5 + 16, 72, "f32")])
def test_linear_vs_fp64(M, N, K, out):
    from respect_b200.kernels.gemm import linear
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    y = linear(x, w, out_dtype=torch.float32 if out == "f32" else None)
    ref = (x.double() @ w.double().T)
    if out == "f32":
        err = (y.double() - ref).abs().max().item()
        assert err < 1e-5 * K ** 0.5 * ref.abs().max().item() + 1e-6
    else:
        assert _bf16_close(y.float().cpu().numpy(), ref.cpu().numpy(), K)


def test_linear_row_count_invariance():
    """The reference's own check (tests/test_kernel_invariance.py:8-17), plus M > 128."""
    from respect_b200.kernels.gemm import linear
    torch.manual_seed(0)
    x = torch.randn(300, 4096, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(1024, 4096, device=DEV, dtype=torch.bfloat16)
    full = linear(x, w)
    for m in (1, 7, 33, 64, 128, 129, 256, 257):
        assert torch.equal(linear(x[:m], w), full[:m])
    # shapes of the 7B model: split-K (o, down) and the wide lm_head
    for (N, K) in ((3584, 3584), (3584, 18944)):
        x = torch.randn(256, K, device=DEV, dtype=torch.bfloat16)
        w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.02
        full = linear(x, w)
        for m in (1, 100, 128, 200):
            assert torch.equal(linear(x[:m], w), full[:m])


@pytest.mark.parametrize("M,N,K", [(128, 4608, 3584), (1, 3584, 18944), (200, 37888, 512), (33, 152064, 256),
                                   (5, 1000, 200)])
def test_linear_packed_is_bitwise_linear(M, N, K):
    from respect_b200.kernels.gemm import linear, linear_packed, pack_weight
    g = torch.Generator(device=DEV).manual_seed(N + K)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    wp = pack_weight(w)
    for od in (None, torch.float32):
        assert torch.equal(linear_packed(x, wp, N, out_dtype=od), linear(x, w, out_dtype=od))


@pytest.mark.parametrize("M,F,K", [(128, 18944, 3584), (1, 18944, 3584), (200, 1024, 512), (5, 384, 200)])
def test_linear_swiglu_packed(M, F, K):
    """Fused gate|up + SiLU*mul: equals eager silu(gate)*up on the same bf16 projections, row-invariant,
    and (7B shape: one split of 256-wide tiles in rb_linear's own plan) bitwise the unfused composition."""
    from respect_b200 import _lib
    from respect_b200.kernels.gemm import (interleave_gate_up, linear, linear_packed, linear_swiglu_packed,
                                           pack_gate_up)
    g = torch.Generator(device=DEV).manual_seed(F + K)
    x = torch.randn(max(M, 2), K, device=DEV, generator=g).to(torch.bfloat16)[:M]
    wg = (torch.randn(F, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(F, K, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    wp = pack_gate_up(wg, wu)
    y = linear_swiglu_packed(x, wp, F)
    assert y.shape == (M, F) and y.dtype == torch.bfloat16
    # row invariance: each row alone gives the same bits
    for r in sorted({0, M // 2, M - 1}):
        assert torch.equal(linear_swiglu_packed(x[r:r + 1], wp, F), y[r:r + 1])
    # against fp64 projections rounded to bf16. A K-long fp32 sum that lands next to a bf16
    # midpoint rounds the other way (one ulp, <= 2^-7 relative, ~0.1% of elements); through
    # silu (gain <= 1.1 for g > 0) and the two later roundings that is up to ~2^-5 relative.
    gr = (x.double() @ wg.double().T).to(torch.bfloat16)
    ur = (x.double() @ wu.double().T).to(torch.bfloat16)
    ref = (torch.nn.functional.silu(gr) * ur).float()
    assert torch.all((y.float() - ref).abs() <= ref.abs() * 2 ** -5 + 1e-4 * ref.abs().max())
    assert (y.float() != ref).float().mean() < 0.01
    N, plan_bn = 2 * F, _lib.lib().rb_linear_bn(2 * F, K)
    if (F, K) == (18944, 3584):
        assert plan_bn == 256
        gu = linear_packed(x, pack_gate_up(wg, wu), N).view(M, F // 128, 2, 128)
        from respect_b200.system.fused import silu_mul
        comp = silu_mul(gu[:, :, 0].reshape(M, F).contiguous(), gu[:, :, 1].reshape(M, F).contiguous())
        assert torch.equal(y, comp)
        assert torch.equal(linear(x, interleave_gate_up(wg, wu)), gu.reshape(M, N))


# ---------------------------------------------------------------- rmsnorm / rope / silu
@pytest.mark.parametrize("N", [128, 384, 3584, 4096])
def test_rmsnorm_vs_oracle_and_row_invariance(N):
    from respect_b200.kernels.rmsnorm import rmsnorm
    rng = np.random.default_rng(N)
    x = round_bf16(rng.standard_normal((64, N), dtype=np.float32))
    w = round_bf16(rng.uniform(0.5, 1.5, N).astype(np.float32))
    y = rmsnorm(T(x, torch.bfloat16), T(w, torch.bfloat16), 1e-6)
    ref = oops.rmsnorm(x, w, 1e-6, bf16=True)
    got = y.float().cpu().numpy()
    # x*rsqrt is rounded to bf16, then w*x̂ again: one-ulp differences in the
    # first rounding (rsqrtf vs exact) can become two ulps in the output.
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2 ** -6 + 1e-7)
    assert (got != ref).mean() < 0.02
    assert torch.equal(rmsnorm(T(x[:1], torch.bfloat16), T(w, torch.bfloat16), 1e-6), y[:1])
    yf = rmsnorm(T(x), T(w), 1e-6)
    assert np.abs(yf.cpu().numpy() - oops.rmsnorm(x, w, 1e-6, bf16=False)).max() < 1e-5


def _rope_eager(q, cos, sin):
    half = q.shape[-1] // 2
    rot = torch.cat([-q[..., half:], q[..., :half]], dim=-1)
    return q * cos[:, None] + rot * sin[:, None]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rope_bitwise_vs_eager(dtype):
    from respect_b200.system.fused import rope
    from respect_b200.decoding.engine import rope_table
    g = torch.Generator(device=DEV).manual_seed(2)
    q = torch.randn(1, 28, 128, 128, device=DEV, generator=g).to(dtype)
    c, s = rope_table(4096, 128, 1e6, DEV)
    pos = 3000 + torch.randint(0, 64, (128,), device=DEV, generator=g)
    cos, sin = c[pos][None].to(dtype), s[pos][None].to(dtype)
    assert torch.equal(rope(q, cos, sin), _rope_eager(q, cos, sin))
    # strided input (a transposed view, as HF passes q)
    qt = torch.randn(1, 128, 28, 128, device=DEV, generator=g).to(dtype).transpose(1, 2)
    assert torch.equal(rope(qt, cos, sin), _rope_eager(qt, cos, sin))


def test_rope_golden_bits():
    from respect_b200.system.fused import rope
    kern = np.load(G / "kernels.npz")
    q = T(from_bf16_bits(kern["rope_q_bits"]), torch.bfloat16)
    cos = T(from_bf16_bits(kern["rope_cos_bits"]), torch.bfloat16)
    sin = T(from_bf16_bits(kern["rope_sin_bits"]), torch.bfloat16)
    out = rope(q, cos, sin).float().cpu().numpy()
    assert np.array_equal(out, from_bf16_bits(kern["rope_out_bits"]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_silu_mul_bitwise_vs_eager(dtype):
    from respect_b200.system.fused import silu_mul
    g = torch.Generator(device=DEV).manual_seed(3)
    a = (torch.randn(128, 18944, device=DEV, generator=g) * 4).to(dtype)
    b = torch.randn(128, 18944, device=DEV, generator=g).to(dtype)
    assert torch.equal(silu_mul(a, b), torch.nn.functional.silu(a) * b)
    assert torch.equal(silu_mul(a[:, :13], b[:, :13]), torch.nn.functional.silu(a[:, :13]) * b[:, :13])


def _eager_rmsnorm(x, w, eps):
    """HF Qwen3-VL RMSNorm forward."""
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return w * (xf * torch.rsqrt(var + eps)).to(x.dtype)


@pytest.mark.parametrize("rdt,hdt", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                     (torch.bfloat16, torch.float32)])
def test_prefill_add_sq_norm_bitwise_vs_eager(rdt, hdt):
    """respect/system/fused.py:126-194: add_sq, norm_from, rmsnorm bit for bit with eager."""
    from respect_b200.system.fused import add_sq, norm_from, rmsnorm
    g = torch.Generator(device=DEV).manual_seed(8)
    r = (torch.randn(300, 3584, device=DEV, generator=g) * 3).to(rdt)
    h = torch.randn(300, 3584, device=DEV, generator=g).to(hdt)
    w = (torch.rand(3584, device=DEV, generator=g) + 0.5).to(torch.bfloat16)
    x, sq = add_sq(r, h)
    assert torch.equal(x, r + h)
    assert torch.equal(sq, (r + h).float() ** 2)
    assert torch.equal(norm_from(x, sq, w, 1e-6), _eager_rmsnorm(r + h, w, 1e-6))
    assert torch.equal(rmsnorm(x, w, 1e-6), _eager_rmsnorm(x, w, 1e-6))
    assert torch.equal(rmsnorm(x, w.float(), 1e-6), _eager_rmsnorm(x, w.float(), 1e-6))


# ---------------------------------------------------------------- decode helpers
def test_greedy_token_matches_masked_argmax():
    from respect_b200.decoding.acceptance import greedy_token, mask_action_vocab
    g = torch.Generator(device=DEV).manual_seed(4)
    lg = torch.randn(130, 152064, device=DEV, generator=g)
    lg[3, 1000:2000] = 50.0           # inside the excluded range: must be skipped
    lg[5, 7] = lg[5, 9] = 60.0        # tie: lowest index wins
    got = greedy_token(lg, 1000, 1000)
    ref = mask_action_vocab(lg, 1000, 1000).argmax(dim=-1)
    assert torch.equal(got, ref)
    assert int(got[5]) == 7
    assert torch.equal(greedy_token(lg.to(torch.bfloat16), 0, 0), lg.to(torch.bfloat16).float().argmax(-1))
    assert np.array_equal(got.cpu().numpy(), otrie.greedy_token(lg.cpu().numpy(), 1000, 1000))


def test_compact_matches_oracle():
    from respect_b200 import _lib
    import ctypes
    rng = np.random.default_rng(6)
    L, HK, S, D = 3, 4, 300, 128
    k = [round_bf16(rng.standard_normal((HK, S, D), dtype=np.float32)) for _ in range(L)]
    v = [round_bf16(rng.standard_normal((HK, S, D), dtype=np.float32)) for _ in range(L)]
    kt = [T(a, torch.bfloat16) for a in k]
    vt = [T(a, torch.bfloat16) for a in v]
    PL, base, path = 200, 4, [0, 2, 3, 7, 8, 20]
    kp = (ctypes.c_void_p * L)(*[t.data_ptr() for t in kt])
    vp = (ctypes.c_void_p * L)(*[t.data_ptr() for t in vt])
    src = (ctypes.c_int32 * len(path))(*[PL + base + p for p in path])
    _lib.call("rb_compact_kv", kp, vp, L, HK, D, S * D, D, 2, src, len(path), PL + base,
              torch.cuda.current_stream().cuda_stream)
    k2, v2 = otrie.compact(k, v, PL, base, path)
    for a, b in zip(kt + vt, k2 + v2):
        assert np.array_equal(a.float().cpu().numpy(), b)


def test_masks_match_golden_and_oracle():
    from respect_b200 import _lib
    z = np.load(G / "verify_mask.npz")
    for i in range(2):
        PL, base, cap, delta = (int(x) for x in z[f"c{i}_meta"])
        parents = T(z[f"c{i}_parents"], torch.int32)
        q = parents.numel()
        m = torch.empty(q, PL + cap, dtype=torch.int16, device=DEV)
        _lib.call("rb_verify_mask", parents.data_ptr(), q, PL + base, PL + cap, m.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        assert np.array_equal(m.cpu().numpy().view(np.uint16), z[f"c{i}_mask_bits"][0, 0])
        committed, MP = 5, ((q + 63) // 64) * 64
        NN = ((committed + q + 31) // 32) * 32
        msk = torch.empty(MP, NN, dtype=torch.uint8, device=DEV)
        _lib.call("rb_trie_node_mask", parents.data_ptr(), q, committed, MP, NN, msk.data_ptr(), NN,
                  torch.cuda.current_stream().cuda_stream)
        allow = np.zeros((q, committed + q), bool)
        allow[:, :committed] = True
        allow[:, committed:] = otrie.ancestry(z[f"c{i}_parents"].tolist())
        _, _, ref = otrie.dispatch_inputs(q, committed + q, allow)
        assert np.array_equal(msk.cpu().numpy().astype(bool), ref[:MP, :NN])


def test_no_device_error_flag():
    from respect_b200 import _lib
    assert _lib.device_error() == 0
