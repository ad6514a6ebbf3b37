"""The candidate sources (datastore, history) against the reference's own outputs.

tests/golden/candidates.json holds what respect.candidates.datastore and
respect.candidates.history returned on seeded sentences (make_golden.py
--only candidates); the known answers below are the reference's own unit
tests (tests/test_trie.py:26-72).
"""
import json
from pathlib import Path

import pytest

from respect_b200.candidates import CocHistory, Datastore, first_token_filter

G = Path(__file__).resolve().parent / "golden"
EOS = 99


@pytest.fixture(scope="module")
def gold():
    return json.loads((G / "candidates.json").read_text())


def _t(xs):
    return [tuple(x) for x in xs]


def test_datastore_matches_reference(gold):
    inp = gold["inputs"]
    checked = 0
    for gmax in (1, 2, 3):
        ds = Datastore(_t(inp["static"]), gmax=gmax).with_drive(_t(inp["drive"]))
        before = {cmax: [ds.lookup(p, cmax) for p in inp["prefixes"]] for cmax in (1, 3, 64)}
        for s in _t(inp["added"]):
            ds.add(s)
        after = {cmax: [ds.lookup(p, cmax) for p in inp["prefixes"]] for cmax in (1, 3, 64)}
        drive_only = {cmax: [ds.without_static().lookup(p, cmax) for p in inp["prefixes"]] for cmax in (1, 3, 64)}
        static = Datastore(_t(inp["static"]), gmax=gmax)
        static_only = {cmax: [static.lookup(p, cmax) for p in inp["prefixes"]] for cmax in (1, 3, 64)}
        ours = {"static+drive": before, "after_add": after, "drive_only": drive_only, "static_only": static_only}
        for rec in gold["lookups"]:
            if rec["gmax"] != gmax:
                continue
            got = [[list(c) for c in outs] for outs in ours[rec["stage"]][rec["cmax"]]]
            assert got == rec["out"], (gmax, rec["stage"], rec["cmax"])
            checked += 1
        assert static.num_entries() == gold["num_entries"][gmax - 1]
    assert checked == 3 * 4 * 3


def test_history_and_first_token_match_reference(gold):
    inp, eos = gold["inputs"], gold["eos"]
    h = CocHistory(eos)
    for f, s in enumerate(inp["frames"]):
        h.append(f, list(s) + [eos] * (f % 3))
        assert [[list(c) for c in h.candidates(n)] for n in range(0, 7)] == gold["history"][f], f
    cands = _t(inp["static"][:20])
    assert [[list(c) for c in first_token_filter(cands, t)] for t in range(10)] == gold["first_token"]


def test_reference_known_answers():
    h = CocHistory(EOS)
    for f, s in enumerate([(1, 2), (3, 4), (1, 2), (5,)]):
        h.append(f, list(s) + [EOS])
    assert h.candidates(3) == [(3, 4, EOS), (1, 2, EOS), (5, EOS)]
    assert first_token_filter([(1, 2), (3, 4)], 3) == [(3, 4)]
    assert first_token_filter([(1, 2)], 7) == [(7,)]
    ds = Datastore([(1, 2, 3, 4), (9, 2, 5)])
    assert ds.lookup([1, 2]) == [(3, 4)]
    assert ds.lookup([7, 2]) == [(3, 4), (5,)]
    assert ds.lookup([42]) == []
    ds = Datastore([(1, 2, 3), (1, 2, 4)]).with_drive([(1, 2, 4)])
    assert ds.lookup([1, 2]) == [(4,), (3,)]
    ds.add((1, 2, 3))
    ds.add((1, 2, 3))
    assert ds.lookup([1, 2]) == [(3,), (4,)]
    assert ds.without_static().lookup([1, 2]) == [(3,), (4,)]
    base = Datastore([(5, 6, 7)])
    d1 = base.with_drive([(5, 6, 8)])
    d1.add((5, 6, 8))
    assert base.lookup([5, 6]) == [(7,)]
    assert base.with_drive([]).lookup([5, 6]) == [(7,)]
