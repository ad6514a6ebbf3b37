"""The oracle (CPU restatement) against fixtures produced by the reference's own code."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import ops, trie as otrie
from oracle.bf16 import from_bf16_bits, round_bf16
from oracle.inputs import attention_case, checksum

G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def kern():
    return np.load(G / "kernels.npz")


def test_round_bf16_ties_to_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf], np.float32)
    # 1 + 2^-8 is exactly halfway between bf16 1.0 and 1.0078125: ties to even -> 1.0
    assert round_bf16(x)[1] == np.float32(1.0)
    assert round_bf16(x)[2] == np.float32(1.015625)
    assert np.isinf(round_bf16(x)[5])


def test_trie_golden():
    cases = json.loads((G / "trie.json").read_text())
    assert len(cases) >= 9
    for c in cases:
        tokens, parents, depths, roots, children, uniq = otrie.build_trie([tuple(s) for s in c["seqs"]])
        assert [[t, p, d] for t, p, d in zip(tokens, parents, depths)] == c["nodes"], c["name"]
        assert [[k, v] for k, v in roots.items()] == c["roots"]
        assert [list(s) for s in uniq] == c["unique"]
        anc = otrie.ancestry(parents)
        assert [np.flatnonzero(anc[i]).tolist() for i in range(len(tokens))] == c["ancestry"]
        for w in c["walks"]:
            tg = {int(k): v for k, v in w["target"].items()}
            path, acc, rec = otrie.walk(roots, tokens, children, w["first"], w["cap"], w["eos"],
                                        lambda a, ch: tg[ch])
            assert (path, acc, rec) == (w["path"], w["acc"], w["rec"]), c["name"]


def test_reference_unit_vectors():
    # tests/test_trie.py of the reference: merge order and ancestry row of node "5"
    tokens, parents, *_ = otrie.build_trie([(1, 2, 3, 99), (1, 2, 4, 99), (1, 2, 3, 99)])
    assert tokens == [1, 2, 3, 99, 4, 99]
    tokens, parents, *_ = otrie.build_trie([(1, 2, 3), (1, 5)])
    assert np.flatnonzero(otrie.ancestry(parents)[3]).tolist() == [0, 3]


def test_verify_mask_golden():
    z = np.load(G / "verify_mask.npz")
    for i in range(2):
        PL, base, cap, delta = z[f"c{i}_meta"]
        parents = z[f"c{i}_parents"].tolist()
        m = otrie.verify_mask(parents, PL, base, cap)
        assert np.array_equal(m, z[f"c{i}_mask_bits"][0, 0])
        slots, logical = otrie.verify_positions(z[f"c{i}_depths"], PL, base, delta)
        assert np.array_equal(slots, z[f"c{i}_cache_position"])
        assert np.array_equal(np.broadcast_to(logical, (3, 1, len(parents))), z[f"c{i}_position_ids"])
        assert np.array_equal(z[f"c{i}_tokens"], z[f"c{i}_ids"][0])


def test_attention_config1_golden(kern):
    c = attention_case(0)
    assert checksum(*[c[k] for k in ("q", "kp", "vp", "kn", "vn", "msk")]) == str(kern["attn_c1_checksum"])
    ref = kern["attn_c1_out"]
    o = oatt.fused_attn_hyb(c["q"], c["kp"], c["vp"], c["kn"], c["vn"], c["msk"])
    assert np.abs(o - ref).max() < 2e-6
    e = oatt.sdpa(c["q"], c["kp"], c["vp"], c["kn"], c["vn"], c["msk"])
    assert np.abs(e - ref).max() < 1e-5  # the reference's kernel vs its eager path


def test_dispatch_golden(kern):
    key, val = kern["disp_kv"]
    PL, base, q_len = 70, 3, 5
    anc = otrie.ancestry([-1, 0, 1, 0, 3])
    query = kern["disp_mask_query"][0]
    n_node = key.shape[2] - PL
    allow = np.zeros((q_len, n_node), bool)
    allow[:, :base] = True
    allow[:, base:base + q_len] = anc
    MP, NN, msk = otrie.dispatch_inputs(q_len, n_node, allow)
    q = np.zeros((query.shape[0], MP, 128), np.float32)
    q[:, :q_len] = query
    kn = np.zeros((key.shape[1], NN, 128), np.float32)
    vn = np.zeros_like(kn)
    kn[:, :n_node] = key[0, :, PL:]
    vn[:, :n_node] = val[0, :, PL:]
    o = oatt.fused_attn_hyb(q, key[0, :, :PL], val[0, :, :PL], kn, vn, msk)
    ref = kern["disp_mask_out"][0]            # [q, H, D]
    assert np.abs(o[:, :q_len].transpose(1, 0, 2) - ref).max() < 2e-6
    # causal (no mask): one token with 6 committed before it
    q1 = kern["disp_causal_query"][0]
    MP, NN, msk = otrie.dispatch_inputs(1, 7, None)
    qq = np.zeros((q1.shape[0], MP, 128), np.float32)
    qq[:, :1] = q1
    kn = np.zeros((key.shape[1], NN, 128), np.float32)
    vn = np.zeros_like(kn)
    kn[:, :7] = key[0, :, PL:PL + 7]
    vn[:, :7] = val[0, :, PL:PL + 7]
    o = oatt.fused_attn_hyb(qq, key[0, :, :PL], val[0, :, :PL], kn, vn, msk)
    assert np.abs(o[:, :1].transpose(1, 0, 2) - kern["disp_causal_out"][0]).max() < 2e-6


def test_linear_rmsnorm_golden(kern):
    y = ops.linear(kern["lin_x"], kern["lin_w"], out_bf16=False)
    assert np.abs(y - kern["lin_y"]).max() < 1e-4
    r = ops.rmsnorm(kern["rms_x"], kern["rms_w"], 1e-6, bf16=False)
    assert np.abs(r - kern["rms_y"]).max() < 1e-5


def test_rope_silu_golden_bitwise(kern):
    q = from_bf16_bits(kern["rope_q_bits"])
    cos = from_bf16_bits(kern["rope_cos_bits"])[:, None]
    sin = from_bf16_bits(kern["rope_sin_bits"])[:, None]
    out = ops.rope(q, cos, sin)
    assert np.array_equal(out, from_bf16_bits(kern["rope_out_bits"]))
    # the oracle's own table reproduces the bf16 cos/sin HF computes
    c, s = ops.rope_cos_sin(np.arange(3000, 3016), 128, 1e6)
    assert np.abs(c - from_bf16_bits(kern["rope_cos_bits"])[0]).max() <= 2 ** -8
    g = from_bf16_bits(kern["silu_g_bits"])
    u = from_bf16_bits(kern["silu_u_bits"])
    ref = from_bf16_bits(kern["silu_out_bits"])
    got = ops.silu_mul(g, u)
    # numpy's float32 exp may differ from ATen's by an ulp before the bf16 rounding
    assert (got != ref).mean() < 0.01
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2 ** -7
