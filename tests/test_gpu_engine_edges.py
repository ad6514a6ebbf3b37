"""Edge cases of the verify engine: malformed or oversized steps are rejected on
the host with the documented status and leave the engine usable; the largest
step (max_rows = 1024, a chain 900 deep) is still bitwise equal to token-by-token
decoding; the device acceptance handles cap 0, an EOS at the root and a first
token held by a later root exactly as the host walk (respect/decoding/acceptance.py:26-46).
"""
import numpy as np
import pytest
import torch

from oracle.inputs import top_up
from respect_b200 import _lib
from respect_b200.candidates.trie import build_trie
from respect_b200.decoding.acceptance import walk
from respect_b200.decoding.engine import DecoderConfig, DecoderWeights, VerifyEngine

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def model():
    cfg = DecoderConfig.tiny(2)
    return cfg, DecoderWeights.random(cfg, DEV, seed=11, std=0.02)


def _status(fn):
    with pytest.raises(_lib.RespectNativeError) as e:
        fn()
    return e.value.status


def test_engine_rejects_malformed_steps(model):
    cfg, w = model
    eng = VerifyEngine(w, max_rows=64, max_slots=256)
    try:
        rng = np.random.default_rng(3)
        P = 100
        eng.prefill(rng.integers(0, cfg.vocab, P))
        tree = build_trie(top_up(rng, [tuple(int(t) for t in rng.integers(0, cfg.vocab, 8))], 40, cfg.vocab))
        ids, par, dep = tree.tokens().astype(np.int32), tree.parents(), tree.depths()
        eng.step(ids, par, dep, 0, P)
        ref = eng.logits(len(ids)).clone()

        bad = par.copy(); bad[5] = 7                      # a parent after its child
        assert _status(lambda: eng.step(ids, bad, dep, 0, P)) == 1
        bad = dep.copy(); bad[5] += 1                      # depth != parent depth + 1
        assert _status(lambda: eng.step(ids, par, bad, 0, P)) == 1
        bad = ids.copy(); bad[3] = cfg.vocab               # token outside the vocabulary
        assert _status(lambda: eng.step(bad, par, dep, 0, P)) == 1
        bad = ids.copy(); bad[3] = -1
        assert _status(lambda: eng.step(bad, par, dep, 0, P)) == 1
        e = np.zeros(0, np.int32)
        assert _status(lambda: eng.step(e, e, e, 0, P)) == 1              # no rows
        big = build_trie(top_up(rng, [(1, 2)], 65, cfg.vocab))          # one row over max_rows
        assert _status(lambda: eng.step(big.tokens().astype(np.int32), big.parents(), big.depths(), 0, P)) == 3
        assert _status(lambda: eng.step(ids, par, dep, 256 - P - len(ids) + 1, P)) == 3  # past max_slots
        assert _status(lambda: eng.step(ids, par, dep, -1, P)) == 1

        # nothing was launched for the rejected calls: the same step gives the same bits
        eng.step(ids, par, dep, 0, P)
        assert torch.equal(eng.logits(len(ids)), ref)
        assert _lib.device_error() == 0
    finally:
        eng.close()


def test_max_rows_step_deep_chain_equals_ar(model):
    """1024 rows (the engine's limit), a 900-token chain among them: the chain's
    greedy picks, logits rows and KV equal 900 one-token steps, bit for bit."""
    cfg, w = model
    P, L = 48, 900
    eng = VerifyEngine(w, max_rows=1024, max_slots=P + 1024 + 8)
    try:
        rng = np.random.default_rng(5)
        eng.prefill(rng.integers(0, cfg.vocab, P))
        toks, rows = [int(rng.integers(0, cfg.vocab))], []
        one_p, one_d = np.array([-1], np.int32), np.array([0], np.int32)
        for t in range(L):
            eng.step(np.array([toks[-1]], np.int32), one_p, one_d, t, P)
            rows.append(eng.logits(1)[0].clone())
            toks.append(int(eng.fetch_ids(1)[0]))
        ar_kv = [(k[:, P:P + L].clone(), v[:, P:P + L].clone()) for k, v in zip(eng.kc, eng.vc)]
        seqs = [tuple(toks[:L])]
        share = 400
        seqs.append(tuple(toks[:share]) + tuple(int(x) for x in rng.integers(0, cfg.vocab, 60)))
        tree = build_trie(top_up(rng, seqs, 1024, cfg.vocab))
        # the chain on nodes in trie order; its slot is PL + node index
        chain = [tree.roots[toks[0]]]
        for t in toks[1:L]:
            chain.append(tree.nodes[chain[-1]].children[t])
        assert len(tree.nodes) == 1024
        eng.step(tree.tokens().astype(np.int32), tree.parents(), tree.depths(), 0, P)
        lg = eng.logits(1024)
        ids = eng.next_ids(1024).cpu().numpy()
        for i, node in enumerate(chain):
            assert torch.equal(lg[node], rows[i]), i
            assert ids[node] == toks[i + 1], i
        for (k, v), (ka, va) in zip(zip(eng.kc, eng.vc), ar_kv):
            idx = torch.tensor([P + n for n in chain], device=k.device)
            assert torch.equal(k[:, idx], ka) and torch.equal(v[:, idx], va)
        # the device acceptance takes the whole chain and moves its KV to consecutive slots
        path, acc, corr = eng.accept(toks[0], 1 << 30, -1)
        assert path == chain and acc == toks[:L] and corr == toks[L]
        for (k, v), (ka, va) in zip(zip(eng.kc, eng.vc), ar_kv):
            assert torch.equal(k[:, P:P + L], ka) and torch.equal(v[:, P:P + L], va)
    finally:
        eng.close()


def test_device_accept_edge_cases(model):
    cfg, w = model
    eng = VerifyEngine(w, max_rows=64, max_slots=256)
    try:
        rng = np.random.default_rng(8)
        P = 40
        eng.prefill(rng.integers(0, cfg.vocab, P))
        # two roots; picks decide the rest
        seqs = [tuple(int(t) for t in rng.integers(0, cfg.vocab, 6)) for _ in range(3)]
        tree = build_trie(top_up(rng, seqs, 30, cfg.vocab))
        args = (tree.tokens().astype(np.int32), tree.parents(), tree.depths(), 0, P)
        roots = list(tree.roots)
        assert len(roots) >= 2
        eng.step(*args)
        picks = eng.fetch_ids(len(tree.nodes))
        pick = lambda a, ch: int(picks[ch])  # noqa: E731
        cases = [(roots[0], 0, -1),            # cap 0: nothing accepted, the correction is `first`
                 (roots[-1], 100, -1),         # `first` held by the last root
                 (roots[0], 100, roots[0]),    # the root itself is EOS: accepted, correction EOS
                 (roots[1], 1, -1)]            # cap 1: the root only
        for first, cap, eos in cases:
            eng.step(*args)
            got = eng.accept(first, cap, eos)
            want = walk(tree, first, cap, eos, pick)
            assert got == (list(want[0]), list(want[1]), want[2]), (first, cap, eos)
        assert eng.accept(roots[0], 0, -1)[2] == roots[0]
    finally:
        eng.close()
