"""Seeded synthetic inputs with the shapes and distributions of BASELINE.json's
configs (the reference's own data — PhysicalAI-AV frames, Alpamayo weights —
are not available; seeded draws stand in for them).

numpy's PCG64 Generator is used so that the same seed gives the same values on
every machine; fixtures record a checksum of their inputs so a drift in the
generator shows up as a clear test failure.
"""
from __future__ import annotations

import hashlib

import numpy as np

from oracle.trie import build_trie


def checksum(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


def chain_seqs(rng, n_chains, length, vocab, max_share=None):
    """n_chains token chains; chain c > 0 shares a seeded prefix with chain 0."""
    max_share = max_share or max(1, length // 2)
    base = [int(t) for t in rng.integers(0, vocab, size=length)]
    seqs = [tuple(base)]
    for _ in range(1, n_chains):
        share = int(rng.integers(1, max_share + 1))
        tail = [int(t) for t in rng.integers(0, vocab, size=length - share)]
        seqs.append(tuple(base[:share] + tail))
    return seqs


def top_up(rng, seqs, target_nodes, vocab):
    """Add seeded sibling leaves (a prefix of an existing sequence plus a new
    token) until the merged trie has exactly target_nodes nodes."""
    seqs = list(seqs)
    while True:
        tokens, parents, depths, roots, children, uniq = build_trie(seqs)
        n = len(tokens)
        if n >= target_nodes:
            return seqs
        s = seqs[int(rng.integers(0, len(seqs)))]
        cut = int(rng.integers(1, len(s) + 1))
        prefix = tuple(s[:cut - 1])
        level = roots
        for t in prefix:
            level = children[level[t]]
        tok = int(rng.integers(0, vocab))
        if tok in level:
            continue
        seqs.append(prefix + (tok,))


def config1_trie(seed=0, vocab=1000):
    """Config 1: 4 seeded chains of 12 tokens merged, topped up to 48 nodes."""
    rng = np.random.default_rng(seed)
    seqs = chain_seqs(rng, 4, 12, vocab)
    return top_up(rng, seqs, 48, vocab)


def attention_case(seed=0, H=28, HK=4, D=128, NP=1536, seqs=None, committed=0):
    """Kernel-level inputs in dispatch layout (dispatch.py:94-115): q [H, M, D]
    with M = number of trie nodes, kp/vp [HK, NP, D], kn/vn [HK, NN, D] with
    NN = committed + nodes rounded up to 32 (zero padding), msk [M, NN] bool
    (committed slots open, then trie ancestry)."""
    from oracle.trie import ancestry
    rng = np.random.default_rng(seed)
    if seqs is None:
        seqs = config1_trie(seed)
    tokens, parents, depths, roots, children, uniq = build_trie(seqs)
    q_n = len(tokens)
    n_node = committed + q_n
    NN = max(32, ((n_node + 31) // 32) * 32)
    q = (rng.standard_normal((H, q_n, D), dtype=np.float32) / np.float32(np.sqrt(D))).astype(np.float32)
    kp = rng.standard_normal((HK, NP, D), dtype=np.float32)
    vp = rng.standard_normal((HK, NP, D), dtype=np.float32)
    kn = np.zeros((HK, NN, D), np.float32)
    vn = np.zeros((HK, NN, D), np.float32)
    kn[:, :n_node] = rng.standard_normal((HK, n_node, D), dtype=np.float32)
    vn[:, :n_node] = rng.standard_normal((HK, n_node, D), dtype=np.float32)
    msk = np.zeros((q_n, NN), bool)
    msk[:, :committed] = True
    msk[:, committed:committed + q_n] = ancestry(parents)
    return dict(q=q, kp=kp, vp=vp, kn=kn, vn=vn, msk=msk, parents=np.array(parents, np.int32),
                depths=np.array(depths, np.int32), tokens=np.array(tokens, np.int64))
