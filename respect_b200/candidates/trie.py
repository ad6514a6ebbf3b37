"""Prefix trie over candidate token sequences.

Same data model and results as ``respect.candidates.trie``
(respect/candidates/trie.py:14-64): `Trie.nodes` in insertion order (a parent
always precedes its children, which the verification kernels rely on),
`Trie.roots` / `Node.children` map a token to a node index, `Trie.seqs` lists
the unique non-empty input sequences in first-seen order.

Adds the flat arrays the device side consumes (`parents`, `depths`,
`tokens`), so a verify step ships three int32 vectors instead of a q x q mask.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Iterable

import numpy as np


@dataclass
class Node:
    token: int
    parent: int | None
    depth: int
    children: OrderedDict = field(default_factory=OrderedDict)


@dataclass
class Trie:
    nodes: list
    roots: OrderedDict
    seqs: list

    def parents(self) -> np.ndarray:
        """int32 [q]: parent index, -1 for a root."""
        return np.fromiter((-1 if n.parent is None else n.parent for n in self.nodes), np.int32, len(self.nodes))

    def depths(self) -> np.ndarray:
        return np.fromiter((n.depth for n in self.nodes), np.int32, len(self.nodes))

    def tokens(self) -> np.ndarray:
        return np.fromiter((n.token for n in self.nodes), np.int64, len(self.nodes))


def _unique(seqs: Iterable) -> list:
    seen: set = set()
    out = []
    for s in seqs:
        t = tuple(s)
        if t and t not in seen:
            seen.add(t)
            out.append(t)
    return out


def build_trie(seqs: Iterable) -> Trie:
    """Merge sequences sharing a prefix into one trie; empty and repeated sequences are dropped."""
    uniq = _unique(seqs)
    nodes: list = []
    roots: OrderedDict = OrderedDict()
    for seq in uniq:
        table, parent = roots, None
        for depth, tok in enumerate(seq):
            idx = table.get(tok)
            if idx is None:
                idx = len(nodes)
                table[tok] = idx
                nodes.append(Node(tok, parent, depth))
            parent = idx
            table = nodes[idx].children
    return Trie(nodes, roots, uniq)


def trie_ancestry(tree: Trie) -> np.ndarray:
    """bool [q, q]: (i, j) is True when node i may attend to node j (j is i or an ancestor)."""
    q = len(tree.nodes)
    allowed = np.zeros((q, q), dtype=np.bool_)
    for i in range(q):
        j: int | None = i
        while j is not None:
            allowed[i, j] = True
            j = tree.nodes[j].parent
    return allowed
