"""The HF drop-in path on the GPU: a Qwen3-VL target verified through
respect_b200's dispatch / patch / FixedKVBuffer / verify_trie / sequential.

The model is make_model_golden.tiny_model(0) (2 layers, hidden 256, 2/1 heads,
head_dim 128) in bf16 on cuda:0, the prompt and trie those of
tests/golden/model.npz. Checked:
  * the trie kernels served every attention call (no rejection, no fallback);
  * logits within the north-star bf16 bar (2e-2 max-abs) of the reference's
    eager path (the same HF model and verify step without the dedicated
    kernels) and of the oracle's bf16 forward, and close to the reference's
    fp32 golden logits;
  * the RESPECT guarantee through HF: the logits and KV of accepted trie nodes
    are bitwise equal to token-by-token decoding with the same kernels, over
    two verification rounds with compaction in between.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

G = Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"
BF16_TOL = 2e-2


class Target:
    def __init__(self, vlm):
        self.vlm = vlm


@pytest.fixture(scope="module")
def hf():
    from tests.golden.make_model_golden import CAP, PL, text_state, tiny_model, weight_checksum
    z = np.load(G / "model.npz")
    vlm = tiny_model(0)
    st = text_state(vlm)
    for k, v in st.items():
        np.testing.assert_allclose(weight_checksum(v), z[f"wsum_{k}"], rtol=1e-6, atol=1e-6, err_msg=k)
    vlm = vlm.to(device=DEV, dtype=torch.bfloat16)
    vlm.model.rope_deltas = torch.zeros(1, 1, dtype=torch.long, device=DEV)
    prompt = torch.from_numpy(z["prompt"]).to(DEV)[None]
    with torch.no_grad():
        pf = vlm(input_ids=prompt, use_cache=True)     # Prefill on the default kernels
    return dict(model=Target(vlm), z=z, st=st, PL=PL, CAP=CAP, prompt=prompt, pf=pf)


def _golden_trie(z):
    from respect_b200.candidates.trie import build_trie
    seqs, o = [], 0
    for n in z["seqs_len"]:
        seqs.append(tuple(int(t) for t in z["seqs_flat"][o:o + n]))
        o += n
    return build_trie(seqs)


def _fresh_buffer(hf):
    from respect_b200.decoding.kv_buffer import FixedKVBuffer
    buf = FixedKVBuffer(hf["PL"], (hf["CAP"],))
    buf.allocate(hf["pf"].past_key_values)
    buf.write_prefill(hf["pf"].past_key_values)
    return buf


def _verify(hf, buf, tree, base=0, dedicated=True):
    from respect_b200.decoding.verify import verify_trie
    from respect_b200.kernels.patch import dedicated_kernels
    cache = buf.window(hf["CAP"])
    args = (hf["model"], {"input_ids": hf["prompt"]}, cache, tree, hf["PL"], base, hf["CAP"])
    if not dedicated:
        return verify_trie(*args)
    with dedicated_kernels(hf["model"], hf["PL"]):
        return verify_trie(*args)


def test_hf_verify_uses_the_trie_kernel(hf):
    from respect_b200.kernels import dispatch
    tree = _golden_trie(hf["z"])
    before = dict(dispatch.STATS)
    _verify(hf, _fresh_buffer(hf), tree)
    torch.cuda.synchronize()
    assert dispatch.STATS["kernel"] - before["kernel"] == 2       # one call per layer
    assert dispatch.STATS["rejected"] == before["rejected"]
    assert dispatch.STATS["fallback"] == 0


def test_hf_verify_matches_reference_eager_and_oracle(hf):
    from oracle import model as omodel
    from oracle.bf16 import round_bf16
    from tests.test_model_golden import TINY_CFG, oracle_weights
    z, PL, CAP = hf["z"], hf["PL"], hf["CAP"]
    tree = _golden_trie(z)
    q = len(tree.nodes)
    buf = _fresh_buffer(hf)
    ours = _verify(hf, buf, tree).logits[0].float()
    k_ours = [bk[0, :, PL:PL + q].float().cpu().numpy() for bk in buf.base_k]
    buf_e = _fresh_buffer(hf)
    eager = _verify(hf, buf_e, tree, dedicated=False).logits[0].float()
    d_eager = (ours - eager).abs().max().item()
    assert d_eager <= BF16_TOL, d_eager
    for li in range(2):
        ke = buf_e.base_k[li][0, :, PL:PL + q].float().cpu().numpy()
        assert np.abs(k_ours[li] - ke).max() <= BF16_TOL * max(1.0, np.abs(ke).max())

    # the oracle's bf16 forward on the same bf16 weights and the same Prefill KV
    W = oracle_weights({k: round_bf16(v) for k, v in hf["st"].items()}, 2, 2, 1, 128)
    kc = [buf.base_k[li][0].float().cpu().numpy().copy() for li in range(2)]
    vc = [buf.base_v[li][0].float().cpu().numpy().copy() for li in range(2)]
    parents = [-1 if n.parent is None else n.parent for n in tree.nodes]
    depths = [n.depth for n in tree.nodes]
    ids = [n.token for n in tree.nodes]
    ref = omodel.verify_step(W, TINY_CFG, ids, parents, depths, PL, 0, kc, vc, bf16=True)
    d_oracle = np.abs(ours.cpu().numpy() - ref).max()
    assert d_oracle <= BF16_TOL, d_oracle
    # the reference's fp32 golden: bf16 weights and activations move logits by a few 1e-3
    d_gold = np.abs(ours.cpu().numpy() - z["logits_dedicated"]).max()
    assert d_gold <= 5 * BF16_TOL, d_gold


def _other(t, V=1000):
    return (t + 1 + V // 2) % V


def test_hf_trie_vs_sequential_bitwise(hf):
    """Two verification rounds with compaction == token-by-token decoding, bitwise."""
    from respect_b200.candidates.trie import build_trie
    from respect_b200.decoding.acceptance import greedy_token, walk
    from respect_b200.decoding.kv_buffer import compact
    from respect_b200.decoding.sequential import forward_tokens, sequential
    from respect_b200.kernels.patch import dedicated_kernels
    model, PL = hf["model"], hf["PL"]
    t0 = int(hf["pf"].logits[0, -1].float().argmax())
    buf = _fresh_buffer(hf)

    # token-by-token with the dedicated kernels: 10 tokens, their logits and KV
    with dedicated_kernels(model, PL):
        chain, _ = sequential(model, buf.view(PL), t0, PL, -1, 0, 0, 10)
        assert len(chain) == 10
        cache, ar_logits = buf.view(PL), []
        for i, t in enumerate(chain):
            cache, lg = forward_tokens(model, torch.tensor([[t]], device=DEV), cache, PL + i)
            ar_logits.append(lg[0, -1])
    ar_k = [layer.keys[0, :, PL:PL + 10] for layer in cache.layers]
    ar_v = [layer.values[0, :, PL:PL + 10] for layer in cache.layers]
    for i in range(9):
        assert int(ar_logits[i].argmax()) == chain[i + 1]

    c = chain
    rounds = [
        (0, [(c[0], _other(c[1]), 7), tuple(c[:5]), (c[0], c[1], _other(c[2])), (_other(c[0]), 3)]),
        (5, [(c[5], _other(c[6])), (c[5], c[6], _other(c[7]), 1), tuple(c[5:10]), (_other(c[5]),)]),
    ]
    win = buf.window(hf["CAP"])
    for base, seqs in rounds:
        tree = build_trie(seqs)
        out = _verify(hf, buf, tree, base=base)
        logits = out.logits[0].float()
        ids = greedy_token(logits, 0, 0).tolist()
        path, acc, rec = walk(tree, c[base], 5, -1, lambda a, node: ids[node])
        assert acc == list(c[base:base + 5]), (acc, c)
        assert path != list(range(5)) or base > 0    # round 0 puts the path on scattered slots
        for j, node in enumerate(path):
            assert torch.equal(logits[node], ar_logits[base + j]), (base, j)
        if base + 5 < 10:
            assert rec == c[base + 5]
        compact(win, PL, base, path)
    torch.cuda.synchronize()
    for li in range(len(ar_k)):
        assert torch.equal(buf.base_k[li][0, :, PL:PL + 10], ar_k[li]), li
        assert torch.equal(buf.base_v[li][0, :, PL:PL + 10], ar_v[li]), li
