"""Token-level parity with the reference (tests/golden/token.npz).

The fixture holds the reference's own verification rounds (its eager path in
fp32 over bf16-valued weights: verify_trie, greedy_token with an excluded
vocabulary range, walk, compact; respect/decoding/verify.py:12-46,
respect/decoding/acceptance.py:11-46, respect/decoding/kv_buffer.py:93-104) on a
4-layer random Qwen3-VL text model, 3 prompts x 2 rounds. `check_rounds` drives
an implementation through the same rounds and compares:

* logits: within the bf16 bar (2e-2 max-abs) of the reference, in full for
  frame 0 round 1 and at the reference's top-8 entries of every node elsewhere;
* the greedy id of every trie node (the accepted-token choice): equal to the
  reference's, except where the reference's own top-2 margin is below the logit
  bar — a near-tie that bf16-level differences may flip, reported as a tie event;
* the acceptance walk (accepted node path, committed tokens, correction token):
  equal to the reference's, or parting from it exactly at a tie event on the path.

Round 2 starts from the reference's round-1 state (the reference's accepted path
is compacted), so every round compares like with like whatever happened before.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

G = Path(__file__).resolve().parent / "golden"
TOL = 2e-2          # the north-star bf16 logit bar; also the tie margin


def load():
    return np.load(G / "token.npz")


def model_state(z):
    """The fixture model's weights (numpy fp32, bf16 values), checked by checksum."""
    import sys
    sys.path.insert(0, str(G))
    from make_model_golden import text_state, weight_checksum
    from make_token_golden import token_model
    st = text_state(token_model(0))
    for k, v in st.items():
        np.testing.assert_allclose(weight_checksum(v), z[f"wsum_{k}"], rtol=1e-6, atol=1e-6, err_msg=k)
    return st


def bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def prefix_kv(z, f, n_layers):
    return [(bits_to_f32(z[f"f{f}_k{li}"]), bits_to_f32(z[f"f{f}_v{li}"])) for li in range(n_layers)]


def _walk(tokens, parents, first, ids):
    """The acceptance walk over a trie given as arrays (respect/decoding/acceptance.py:26-46;
    no EOS, no cap, as the fixture ran it)."""
    roots, children = {}, {}
    for i, (t, p) in enumerate(zip(tokens, parents)):
        (roots if p < 0 else children.setdefault(int(p), {}))[int(t)] = i
    path, acc, rec = [], [], first
    ch = roots.get(first)
    while ch is not None:
        path.append(ch)
        acc.append(int(tokens[ch]))
        rec = int(ids[ch])
        ch = children.get(ch, {}).get(rec)
    return path, acc, rec


def check_rounds(z, run_round, reset_frame, compact):
    """Drive an implementation through the fixture's rounds.

    reset_frame(f): load frame f's prefix KV (slots [0, PL)) and clear the rest.
    run_round(tokens, parents, depths, base, act_off, act_size) -> (logits [q, V] fp32 numpy,
        greedy ids [q] with the excluded range masked).
    compact(path, base): move the path's KV to slots PL + base + i.
    Returns a report dict; raises AssertionError on a parity failure."""
    PL, CAP, OFF, SIZE, FRAMES = (int(x) for x in z["meta"])
    report = dict(nodes=0, equal=0, ties=[], walks=0, walks_equal=0, committed_equal=0, max_abs=0.0)
    for f in range(FRAMES):
        reset_frame(f)
        for r in (1, 2):
            p = f"f{f}_r{r}_"
            tokens, parents, depths = z[p + "tokens"], z[p + "parents"], z[p + "depths"]
            base, first, rec_ref = (int(x) for x in z[p + "meta"])
            lg, ids = run_round(tokens, parents, depths, base, OFF, SIZE)
            lg = np.asarray(lg, np.float32)
            ids = np.asarray(ids).astype(np.int64)
            if p + "logits" in z.files:
                d = float(np.abs(lg - z[p + "logits"]).max())
            else:
                at = np.take_along_axis(lg, z[p + "top8_idx"].astype(np.int64), 1)
                d = float(np.abs(at - z[p + "top8_val"]).max())
            report["max_abs"] = max(report["max_abs"], d)
            assert d <= TOL, f"frame {f} round {r}: logits differ by {d} > {TOL}"
            ref_ids = z[p + "greedy"]
            margin = z[p + "top8_val"][:, 0] - z[p + "top8_val"][:, 1]
            report["nodes"] += len(ids)
            tie_nodes = set()
            for n in np.flatnonzero(ids != ref_ids):
                assert margin[n] < TOL, (f"frame {f} round {r} node {n}: greedy id {ids[n]} != reference "
                                         f"{ref_ids[n]} with reference top-2 margin {margin[n]:.4g} >= {TOL}")
                tie_nodes.add(int(n))
                report["ties"].append(dict(frame=f, round=r, node=int(n), ours=int(ids[n]), ref=int(ref_ids[n]),
                                           margin=float(margin[n])))
            report["equal"] += int((ids == ref_ids).sum())
            path, acc, rec = _walk(tokens, parents, first, ids)
            ref_path, ref_acc = z[p + "path"].tolist(), z[p + "acc"].tolist()
            report["walks"] += 1
            if (path, acc, rec) == (ref_path, ref_acc, rec_ref):
                report["walks_equal"] += 1
                report["committed_equal"] += len(acc)
            else:
                # the walks may part only after a node of the shared path that is a tie event
                k = 0
                while k < min(len(path), len(ref_path)) and path[k] == ref_path[k]:
                    k += 1
                last = ref_path[k - 1] if k > 0 else None
                assert last is not None and last in tie_nodes, (
                    f"frame {f} round {r}: walk differs at depth {k} without a tie ({path} vs {ref_path})")
                report["committed_equal"] += k
            compact(ref_path, base)
    return report


def committed_total(z):
    return sum(len(z[f"f{f}_r{r}_acc"]) for f in range(int(z["meta"][4])) for r in (1, 2))
