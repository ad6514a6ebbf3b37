"""Candidate structures and sources for trie verification (mirror of ``respect.candidates``)."""
from respect_b200.candidates.datastore import Datastore
from respect_b200.candidates.history import CocHistory, first_token_filter, strip_eos, unique_recent
from respect_b200.candidates.trie import Node, Trie, build_trie, trie_ancestry

__all__ = ["Node", "Trie", "build_trie", "trie_ancestry", "Datastore", "CocHistory", "first_token_filter",
           "strip_eos", "unique_recent"]
