"""RESPECT decoding on the native engine reproduces token-by-token decoding.

The guarantee RESPECT is built on (respect/decoding/respect.py:1-14): with the
dedicated kernels, the tokens and the KV of a decode equal `sequential` under the
same kernels, whatever the candidates. Checked on a 2-layer random model with
history candidates that hold part of the model's own continuation (long initial
acceptance), with none (one token per round), with an EOS in the middle and with
the sequential follow-up.
"""
import numpy as np
import pytest
import torch

from respect_b200.candidates.datastore import Datastore
from respect_b200.candidates.history import CocHistory
from respect_b200.decoding.engine import DecoderConfig, DecoderWeights, VerifyEngine
from respect_b200.decoding.respect import FrameState, RespectDecoder, sequential

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = 64
MAXT = 48


@pytest.fixture(scope="module")
def setup():
    cfg = DecoderConfig.tiny(2)
    w = DecoderWeights.random(cfg, DEV, seed=2, std=0.02)
    eng = VerifyEngine(w, max_rows=128, max_slots=1024)
    rng = np.random.default_rng(12)
    eng.prefill(rng.integers(0, cfg.vocab, P))
    first = int(rng.integers(0, cfg.vocab))
    yield cfg, eng, rng, first
    eng.close()


def _kv(eng, n):
    return [(k[:, P:P + n].clone(), v[:, P:P + n].clone()) for k, v in zip(eng.kc, eng.vc)]


def _same_kv(a, b):
    return all(torch.equal(x, y) and torch.equal(u, v) for (x, u), (y, v) in zip(a, b))


def test_decode_equals_sequential(setup):
    cfg, eng, rng, first = setup
    fs = FrameState(P, first, MAXT)
    ref = sequential(eng, fs, first, 0, -1, MAXT)
    assert len(ref) == MAXT
    ref_kv = _kv(eng, MAXT)
    dec = RespectDecoder(eng, eos=-1)

    # previous CoCs: the first 20 tokens of the true continuation and two distractors
    distract = [tuple([first] + [int(t) for t in rng.integers(0, cfg.vocab, 15)]) for _ in range(2)]
    res = dec.decode(fs, [tuple(ref[:20])] + distract, Datastore([tuple(ref)]))
    assert res.tokens == ref
    assert res.accepted_initial == 20 and res.target_runs < MAXT
    assert _same_kv(_kv(eng, MAXT), ref_kv)

    # no candidates, empty datastore: one token per target run
    res = dec.decode(fs, [], None)
    assert res.tokens == ref and res.target_runs == MAXT and res.initial_nodes == 1
    assert _same_kv(_kv(eng, MAXT), ref_kv)

    # the rest token by token after the initial verification
    res = dec.decode(fs, [tuple(ref[:10])], None, follow="sequential")
    assert res.tokens == ref and res.accepted_initial == 10
    assert _same_kv(_kv(eng, MAXT), ref_kv)


def test_decode_stops_at_eos(setup):
    cfg, eng, rng, first = setup
    fs = FrameState(P, first, MAXT)
    full = sequential(eng, fs, first, 0, -1, MAXT)
    eos = full[30]
    ref = sequential(eng, fs, first, 0, eos, MAXT)
    assert ref[-1] == eos and len(ref) <= 31
    hist = CocHistory(eos)
    hist.append(0, ref)                       # last frame's CoC: candidates end with EOS
    res = RespectDecoder(eng, eos=eos).decode(fs, hist.candidates(4), Datastore([tuple(full)]))
    assert res.tokens == ref
