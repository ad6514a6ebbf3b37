"""RespectDecoder's loop on the host, with an engine stand-in (no GPU).

The stand-in's greedy pick after a token is a fixed bigram function, so the
verification of a trie and the acceptance walk (respect/decoding/acceptance.py:26-46,
restated over the step's arrays) are exact host computations. The decoder's own logic
is what is tested (respect/decoding/respect.py:86-188): first-token filtering
of the previous CoCs, datastore follow-ups trimmed to the room left, the node
budget, EOS and max_tokens. Its tokens must equal token-by-token decoding with
the same stand-in (respect/decoding/sequential.py:26-42).
"""
import numpy as np

from respect_b200.candidates.datastore import Datastore
from respect_b200.candidates.history import CocHistory
from respect_b200.decoding.respect import FrameState, RespectConfig, RespectDecoder, sequential

V = 97


def pick(tok: int) -> int:
    return (tok * 31 + 7) % V


class BigramEngine:
    """Engine interface of VerifyEngine (step / accept / fetch_ids) over a bigram model."""
    device = "cpu"
    max_rows = 256

    def __init__(self):
        self.steps = 0
        self.rows = []

    def step(self, ids, parents, depths, base, prompt_len, rope_delta=0, act_off=0, act_size=0, **kw):
        ids, parents, depths = (np.asarray(a) for a in (ids, parents, depths))
        assert ids.shape == parents.shape == depths.shape and len(ids) <= self.max_rows
        assert all(parents[i] < i for i in range(len(ids)))
        self.ids, self.parents = ids.astype(int), parents.astype(int)
        self.picks = np.array([pick(int(t)) for t in self.ids])
        self.steps += 1
        self.rows.append(len(ids))

    def fetch_ids(self, q=None):
        return self.picks[:q]

    def accept(self, first, cap, eos, n=None, stream=None):
        """The acceptance walk over the step's arrays: from the root holding `first`,
        while the child holding the pick after its parent exists, up to `cap` tokens,
        stopping after EOS; the correction is the last pick (`first` if nothing matched)."""
        children: dict = {}
        for i, p in enumerate(self.parents):
            children.setdefault(int(p), {})[int(self.ids[i])] = i
        path, acc, corr = [], [], first
        node = children.get(-1, {}).get(first)
        while node is not None and len(acc) < cap:
            path.append(node)
            acc.append(int(self.ids[node]))
            if acc[-1] == eos:
                break
            corr = int(self.picks[node])
            node = children.get(node, {}).get(corr)
        return path, acc, corr


def truth(first, n):
    out = [first]
    while len(out) < n:
        out.append(pick(out[-1]))
    return out


def test_decode_equals_sequential_with_history_and_datastore():
    eng = BigramEngine()
    first = 5
    ref = sequential(eng, FrameState(10, first, 40), first, 0, -1, 40)
    assert ref == truth(first, 40)
    dec = RespectDecoder(eng, eos=-1, cfg=RespectConfig(node_budget=16))
    # previous CoCs: part of the true continuation, a distractor with the same first token
    # and one with another first token (dropped by the filter)
    cocs = [tuple(ref[:12]), (first, 1, 2, 3), (6, 6, 6)]
    ds = Datastore([tuple(ref[10:40])])
    eng.steps = 0
    res = dec.decode(FrameState(10, first, 40), cocs, ds)
    assert res.tokens == ref
    assert res.accepted_initial == 12 and res.target_runs == 1 + res.follow_rounds
    assert res.target_runs < 40 and eng.steps == res.target_runs
    assert max(eng.rows[-res.target_runs:]) <= 16 + 1   # follow-up tries within the node budget
    # no candidates: one token per round
    eng.steps = 0
    res = dec.decode(FrameState(10, first, 40), [], None)
    assert res.tokens == ref and res.target_runs == 40
    # the sequential follow-up
    res = dec.decode(FrameState(10, first, 40), [tuple(ref[:7])], None, follow="sequential")
    assert res.tokens == ref and res.accepted_initial == 7 and res.target_runs == 1 + 33


def test_decode_stops_at_eos_and_max_tokens():
    eng = BigramEngine()
    first = 11
    full = truth(first, 30)
    eos = full[17]
    ref = sequential(eng, FrameState(4, first, 30), first, 0, eos, 30)
    assert ref == full[:18] and ref[-1] == eos
    h = CocHistory(eos)
    h.append(0, ref)                                   # last frame's CoC, EOS appended by the history
    res = RespectDecoder(eng, eos=eos).decode(FrameState(4, first, 30), h.candidates(4), Datastore.empty())
    assert res.tokens == ref and res.target_runs == 1
    # max_tokens cuts a fully matching candidate
    res = RespectDecoder(eng, eos=-1).decode(FrameState(4, first, 9), [tuple(full)], None)
    assert res.tokens == full[:9] and res.target_runs == 1
