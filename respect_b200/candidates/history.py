"""Initial candidates: the CoCs completed in the previous frames of a drive.

Same behaviour as ``respect.candidates.history`` (respect/candidates/history.py:1-50):
the history keeps (frame, CoC without trailing EOS) in frame order;
`candidates(n)` returns the distinct non-empty CoCs of the last n frames, the
newest occurrence of each kept and the order by that occurrence, each with EOS
appended; `first_token_filter` keeps the sentences that start with the token
Prefill fixed (or the single-token sentence when none does).

Host code: the candidate source of the initial verification.
"""
from __future__ import annotations

from typing import Iterable


def strip_eos(tokens: Iterable[int], eos: int) -> tuple[int, ...]:
    out = [int(t) for t in tokens]
    while out and out[-1] == eos:
        del out[-1]
    return tuple(out)


def unique_recent(entries: list, n: int) -> list:
    """(frame, CoC) pairs of the last n entries, the newest of each distinct non-empty CoC, in frame order."""
    window = entries[-n:]                # as list slicing has it: n = 0 keeps every entry
    newest: dict = {}
    for pos, (_, coc) in enumerate(window):
        if coc:
            newest[coc] = pos          # the last position wins
    keep = sorted(newest.values())
    return [window[pos] for pos in keep]


class CocHistory:
    """Rolling record of the CoCs produced by previous frames of one drive."""

    def __init__(self, eos: int) -> None:
        self.eos = eos
        self.entries: list = []

    def append(self, frame_idx: int, tokens: Iterable[int]) -> None:
        self.entries.append((frame_idx, strip_eos(tokens, self.eos)))

    def candidates(self, n: int) -> list[tuple[int, ...]]:
        """Distinct CoCs of the last n frames, each terminated by EOS."""
        return [coc + (self.eos,) for _, coc in unique_recent(self.entries, n)]


def first_token_filter(candidates: list, first: int) -> list:
    """Sentences starting with `first`; the single-token sentence when there is none."""
    keep = [s for s in candidates if s and s[0] == first]
    return keep if keep else [(first,)]
