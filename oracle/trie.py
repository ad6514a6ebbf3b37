"""Trie construction, ancestry, masks, greedy choice, acceptance walk and KV
compaction, restated in plain Python/numpy.

* `build_trie`        respect/candidates/trie.py:31-48 — unique non-empty
                      sequences in first-seen order, merged on shared
                      prefixes; new nodes appended, so parents precede children.
* `ancestry`          respect/candidates/trie.py:51-64 — (i, j) true iff j is
                      i or an ancestor of i.
* `verify_mask`       respect/decoding/verify.py:35-41 — additive bf16 mask
                      [q, PL+cap]: 0 before start = PL+base, ancestry inside the
                      trie window, bf16 lowest elsewhere.
* `verify_positions`  respect/decoding/verify.py:24-33 — slots PL+base+i,
                      rotary positions PL+base+depth+rope_delta.
* `dispatch_inputs`   respect/kernels/dispatch.py:94-115 — rows padded to a
                      multiple of 64, nodes to a multiple of 32, padding rows
                      open node 0, causal mask when no 4-D mask is given.
* `greedy_token`      respect/decoding/acceptance.py:11-23.
* `walk`              respect/decoding/acceptance.py:26-46.
* `compact`           respect/decoding/kv_buffer.py:93-104.
"""
from __future__ import annotations

import numpy as np

BF16_LOWEST_BITS = 0xFF7F


def build_trie(seqs):
    """Returns (tokens, parents, depths, roots: dict token->node, children: list of dicts)."""
    uniq = []
    for s in seqs:
        s = tuple(s)
        if len(s) and s not in uniq:
            uniq.append(s)
    tokens, parents, depths, children = [], [], [], []
    roots = {}
    for s in uniq:
        level, parent = roots, -1
        for d, t in enumerate(s):
            if t not in level:
                level[t] = len(tokens)
                tokens.append(int(t))
                parents.append(parent)
                depths.append(d)
                children.append({})
            parent = level[t]
            level = children[parent]
    return tokens, parents, depths, roots, children, uniq


def ancestry(parents):
    q = len(parents)
    a = np.zeros((q, q), bool)
    for i in range(q):
        j = i
        while j >= 0:
            a[i, j] = True
            j = parents[j]
    return a


def verify_mask(parents, prompt_len, base, capacity):
    """uint16 bf16 bit patterns [q, prompt_len + capacity]."""
    q = len(parents)
    start = prompt_len + base
    m = np.full((q, prompt_len + capacity), BF16_LOWEST_BITS, np.uint16)
    m[:, :start] = 0
    anc = ancestry(parents)
    m[:, start:start + q] = np.where(anc, 0, BF16_LOWEST_BITS)
    return m


def verify_positions(depths, prompt_len, base, rope_delta=0):
    q = len(depths)
    start = prompt_len + base
    slots = np.arange(start, start + q)
    logical = np.asarray(depths, np.int64) + start + rope_delta
    return slots, logical


def dispatch_inputs(q_len, n_node, node_allow=None):
    """(MP, NN, msk [MP, NN] bool) as dispatch.unified_forward builds them."""
    MP = ((q_len + 63) // 64) * 64
    NN = max(32, ((max(n_node, 1) + 31) // 32) * 32)
    msk = np.zeros((MP, NN), bool)
    if node_allow is not None:
        msk[:q_len, :n_node] = node_allow
    else:
        first = n_node - q_len
        rows = np.arange(q_len)[:, None] + first
        msk[:q_len, :] = np.arange(NN)[None, :] <= rows
    msk[q_len:, 0] = True
    return MP, NN, msk


def greedy_token(logits, offset, size):
    x = np.asarray(logits, np.float32).copy()
    x[:, offset:offset + size] = -np.inf
    return x.argmax(axis=-1)


def walk(roots, tokens, children, first, cap, eos, pick):
    path, acc = [], []
    node, rec = roots.get(first), first
    while node is not None and len(acc) < cap:
        path.append(node)
        acc.append(tokens[node])
        if tokens[node] == eos:
            break
        rec = pick(acc, node)
        node = children[node].get(rec)
    return path, acc, rec


def compact(k, v, prompt_len, base, slots):
    """k, v: [HK, S, D] arrays per layer (lists). Returns new copies."""
    if not len(slots):
        return [x.copy() for x in k], [x.copy() for x in v]
    src = np.array([prompt_len + base + s for s in slots])
    dst = np.arange(prompt_len + base, prompt_len + base + len(slots))
    k2, v2 = [], []
    for a, b in zip(k, v):
        a, b = a.copy(), b.copy()
        a[:, dst] = a[:, src].copy()
        b[:, dst] = b[:, src].copy()
        k2.append(a)
        v2.append(b)
    return k2, v2
