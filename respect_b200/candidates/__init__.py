"""Candidate structures for trie verification (mirror of ``respect.candidates``)."""
from respect_b200.candidates.trie import Node, Trie, build_trie, trie_ancestry

__all__ = ["Node", "Trie", "build_trie", "trie_ancestry"]
