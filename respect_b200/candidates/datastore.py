"""Datastore of completed CoCs, searched by the last committed tokens.

Same behaviour as ``respect.candidates.datastore`` (respect/candidates/datastore.py:1-73):
two indexes (static: CoCs of other drives, built once; drive: CoCs completed
earlier in this drive, grown with `add`), each mapping a key of the last g
tokens (g = gmax .. 1) to the counts of the continuations that followed it (to
the end of the stored sentence). A lookup tries the longest key first, falls
back to shorter ones on a miss, adds the two indexes' counts and returns the
continuations most frequent first; equal counts keep first-seen order, static
index first.

Host code: the candidate source of the follow-up verification loop.
"""
from __future__ import annotations

from typing import Iterable


class _Index:
    """key length g -> {key tuple: {continuation tuple: count}} (dicts keep first-seen order)."""

    def __init__(self, gmax: int, seqs: Iterable = ()) -> None:
        self.gmax = gmax
        self.by_len: list[dict] = [dict() for _ in range(gmax + 1)]
        for s in seqs:
            self.add(tuple(s))

    def add(self, s: tuple) -> None:
        n = len(s)
        for g in range(1, self.gmax + 1):
            table = self.by_len[g]
            for i in range(n - g):          # a key is followed by at least one token
                conts = table.setdefault(s[i:i + g], {})
                cont = s[i + g:]
                conts[cont] = conts.get(cont, 0) + 1

    def get(self, key: tuple) -> dict | None:
        return self.by_len[len(key)].get(key)


class Datastore:
    def __init__(self, static_seqs: Iterable = (), gmax: int = 2, drive_seqs: Iterable = ()) -> None:
        self.gmax = gmax
        self.static = _Index(gmax, static_seqs)
        self.drive = _Index(gmax, drive_seqs)

    @classmethod
    def empty(cls, gmax: int = 2) -> "Datastore":
        return cls((), gmax=gmax)

    def _derive(self, static: _Index, drive: _Index) -> "Datastore":
        ds = Datastore.__new__(Datastore)
        ds.gmax, ds.static, ds.drive = self.gmax, static, drive
        return ds

    def with_drive(self, drive_seqs: Iterable) -> "Datastore":
        """Same static index (shared, never modified), a fresh drive index from `drive_seqs` in order."""
        return self._derive(self.static, _Index(self.gmax, drive_seqs))

    def without_static(self) -> "Datastore":
        """The drive index alone."""
        return self._derive(_Index(self.gmax), self.drive)

    def add(self, seq) -> None:
        """One completed CoC into the drive index."""
        self.drive.add(tuple(seq))

    def lookup(self, prefix: list, cmax: int = 64) -> list[tuple]:
        """Continuations after the longest matching key of `prefix`, most frequent first."""
        for g in range(min(self.gmax, len(prefix)), 0, -1):
            key = tuple(prefix[-g:])
            a, b = self.static.get(key), self.drive.get(key)
            if not a and not b:
                continue
            merged = dict(a) if a else {}
            for cont, n in (b or {}).items():
                merged[cont] = merged.get(cont, 0) + n
            # stable sort: equal counts keep first-seen order
            ranked = sorted(merged.items(), key=lambda kv: -kv[1])
            return [cont for cont, _ in ranked[:cmax]]
        return []

    def num_entries(self) -> int:
        """Distinct (key, continuation) pairs of the static index at the longest key length."""
        return sum(len(conts) for conts in self.static.by_len[self.gmax].values())
