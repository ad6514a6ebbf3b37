"""The oracle's verify forward against the reference's own full-model verify step.

tests/golden/model.npz holds what respect.decoding.verify.verify_trie returned
(fp32, CPU, reference kernels interpreted) on a 2-layer random Qwen3-VL text
model built by make_model_golden.tiny_model(0). The oracle restates that
forward in numpy; here it must reproduce the reference's logits and node KV
within the fp32 bar of 1e-5 max-abs.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import model as omodel
from oracle import trie as otrie

G = Path(__file__).resolve().parent / "golden"
FP32_TOL = 1e-5


@pytest.fixture(scope="module")
def gold():
    return np.load(G / "model.npz")


@pytest.fixture(scope="module")
def tiny(gold):
    from tests.golden.make_model_golden import text_state, tiny_model, weight_checksum
    st = text_state(tiny_model(0))
    for k, v in st.items():
        np.testing.assert_allclose(weight_checksum(v), gold[f"wsum_{k}"], rtol=1e-6, atol=1e-6, err_msg=k)
    return st


def oracle_weights(st, n_layers, H, HK, D):
    layers = [dict(wq=st[f"l{i}_q"], wk=st[f"l{i}_k"], wv=st[f"l{i}_v"], wo=st[f"l{i}_o"],
                   wg=st[f"l{i}_g"], wu=st[f"l{i}_u"], wd=st[f"l{i}_d"], in_norm=st[f"l{i}_in"],
                   post_norm=st[f"l{i}_post"], q_norm=st[f"l{i}_qn"], k_norm=st[f"l{i}_kn"])
              for i in range(n_layers)]
    return dict(embed=st["embed"], lm_head=st["lm_head"], final_norm=st["final_norm"], layers=layers)


TINY_CFG = dict(n_heads=2, n_kv_heads=1, head_dim=128, rms_eps=1e-6, rope_theta=1e6)


def test_trie_matches_reference(gold):
    lens = gold["seqs_len"]
    flat = gold["seqs_flat"].tolist()
    seqs, o = [], 0
    for n in lens:
        seqs.append(tuple(flat[o:o + n]))
        o += n
    tokens, parents, depths, *_ = otrie.build_trie(seqs)
    assert tokens == gold["trie_tokens"].tolist()
    assert parents == gold["trie_parents"].tolist()
    assert depths == gold["trie_depths"].tolist()


def test_reference_kernel_path_was_taken(gold):
    # the dedicated run went through the reference's trie kernel in both layers, with no fallback
    assert gold["stats_dedicated"].tolist() == [2, 0]
    np.testing.assert_allclose(gold["logits_dedicated"], gold["logits_eager"], atol=FP32_TOL, rtol=0)


@pytest.mark.parametrize("which", ["eager", "dedicated"])
def test_oracle_verify_matches_reference(gold, tiny, which):
    PL, CAP = (int(x) for x in gold["meta"])
    parents, depths = gold["trie_parents"], gold["trie_depths"]
    q = len(parents)
    W = oracle_weights(tiny, 2, 2, 1, 128)
    kc, vc = [], []
    for li in range(2):
        k = np.zeros((1, PL + CAP, 128), np.float32)
        v = np.zeros_like(k)
        k[:, :PL] = gold[f"k{li}_{which}"][:, :PL]   # the Prefill KV the reference wrote
        v[:, :PL] = gold[f"v{li}_{which}"][:, :PL]
        kc.append(k)
        vc.append(v)
    logits = omodel.verify_step(W, TINY_CFG, gold["trie_tokens"], parents, depths, PL, 0, kc, vc, bf16=False)
    ref = gold[f"logits_{which}"]
    assert logits.shape == ref.shape == (q, 1000)
    np.testing.assert_allclose(logits, ref, atol=FP32_TOL, rtol=0)
    for li in range(2):
        np.testing.assert_allclose(kc[li][:, PL:PL + q], gold[f"k{li}_{which}"][:, PL:], atol=FP32_TOL, rtol=0)
        np.testing.assert_allclose(vc[li][:, PL:PL + q], gold[f"v{li}_{which}"][:, PL:], atol=FP32_TOL, rtol=0)
    # the greedy choices agree wherever the reference's top-2 margin exceeds the tolerance
    top2 = np.sort(ref, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 2 * FP32_TOL
    assert np.array_equal(logits.argmax(1)[clear], ref.argmax(1)[clear])
