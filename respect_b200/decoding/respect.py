"""RESPECT decoding on the native verify engine.

Mirror of ``respect.decoding.respect.RespectDecoder`` (respect/decoding/respect.py:64-188)
and ``respect.config.RespectConfig`` (respect/config.py:10-19), driving
`VerifyEngine` instead of the HF target: initial verification of the previous
CoCs (first-token filtered, one trie, one verify step), then follow-up
verification rounds whose tries hold the datastore's continuations of the
committed tokens (trimmed to the room left, deduplicated, kept while the merged
trie stays within the node budget) until EOS or `max_tokens`. Every verify step
is the engine's graph-captured step (one graph per power-of-two row bucket);
the acceptance walk and the KV compaction run on the device
(`VerifyEngine.accept`). The FD-DFlash drafter of the reference is not part of
this build: the follow-up candidates come from the datastore alone (the
reference's `use_draft=False` path).

`sequential` is the token-by-token reference on the same engine (1-node
verify steps), the output RESPECT must reproduce (respect/decoding/sequential.py:26-42).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from respect_b200.candidates.datastore import Datastore
from respect_b200.candidates.history import first_token_filter
from respect_b200.candidates.trie import build_trie
from respect_b200.decoding.engine import VerifyEngine


@dataclass(frozen=True)
class RespectConfig:
    num_prev_frames: int = 4          # previous frames whose CoCs form the initial trie
    node_budget: int = 64             # nodes per follow-up trie
    draft_tree_nodes: int = 16        # (drafter settings, kept for interface parity)
    draft_topk: int = 4
    datastore_key_len: int = 2        # longest datastore key; shortened to 1 on a miss
    follow_capacity: int = 192        # slots after the prompt used by follow-up verification
    buffer_capacities: tuple = (192, 256, 512, 1024)
    max_new_tokens: int = 128


@dataclass
class FrameState:
    """One frame after Prefill: the prompt KV is in the engine's slots [0, prompt_len)."""
    prompt_len: int
    first_token: int
    max_tokens: int
    rope_delta: int = 0


@dataclass
class DecodeResult:
    tokens: list
    target_runs: int
    accepted_initial: int
    initial_nodes: int
    initial_candidates: int
    follow_rounds: int = 0
    round_nodes: list = field(default_factory=list)
    round_accepted: list = field(default_factory=list)
    initial_ms: float = 0.0
    follow_ms: float = 0.0
    lookup_ms: float = 0.0
    datastore_insert_ms: float = 0.0
    verify_ms: float = 0.0


def _sync(device) -> None:
    """Wait for the device's queued work (timing fields); nothing to wait for off CUDA."""
    if torch.device(device).type == "cuda":
        torch.cuda.synchronize(device)


def _fit(capacities, n: int) -> int:
    for c in sorted(capacities):
        if c >= n:
            return c
    raise ValueError(f"no capacity holds {n} slots (capacities {tuple(capacities)})")


class RespectDecoder:
    def __init__(self, engine: VerifyEngine, eos: int, cfg: RespectConfig = RespectConfig(),
                 act_off: int = 0, act_size: int = 0) -> None:
        self.eng = engine
        self.eos = eos
        self.cfg = cfg
        self.act = (act_off, act_size)

    def _verify(self, fs: FrameState, tree, base: int, first: int, cap: int):
        """One verify step over `tree` after `base` committed tokens; device walk + compaction."""
        q = len(tree.nodes)
        if q > self.eng.max_rows:
            raise ValueError(f"trie of {q} nodes exceeds the engine's max_rows {self.eng.max_rows}")
        self.eng.step(tree.tokens().astype(np.int32), tree.parents(), tree.depths(), base, fs.prompt_len,
                      rope_delta=fs.rope_delta, act_off=self.act[0], act_size=self.act[1])
        return self.eng.accept(first, cap, self.eos, n=q)

    def _initial(self, fs: FrameState, candidates: list):
        cands = first_token_filter(candidates, fs.first_token)
        tree = build_trie(cands)
        path, acc, rec = self._verify(fs, tree, 0, fs.first_token, fs.max_tokens)
        return acc, rec, len(tree.nodes), len(cands)

    def _follow(self, fs: FrameState, committed: list, root: int, datastore: Datastore, res: DecodeResult) -> list:
        cfg = self.cfg
        capacity = _fit(cfg.buffer_capacities, max(cfg.follow_capacity, fs.max_tokens + cfg.node_budget))
        tokens, cur = list(committed), root
        cap_ = fs.max_tokens
        while True:
            base = len(tokens)
            if base >= cap_ or base >= capacity:
                return tokens
            room = min(cap_, capacity) - base
            t1 = time.perf_counter()
            order = [tuple([cur] + [int(x) for x in g]) for g in datastore.lookup(tokens + [cur])]
            cands: list = []
            for seq in order:
                seq = seq[:room]
                if not seq or seq in cands:
                    continue
                if len(build_trie(cands + [seq]).nodes) > cfg.node_budget:
                    continue
                cands.append(seq)
            if not cands:
                cands = [(cur,)]
            tree = build_trie(cands)
            t2 = time.perf_counter()
            path, accepted, recovery = self._verify(fs, tree, base, cur, cap_ - base)
            t3 = time.perf_counter()
            res.lookup_ms += (t2 - t1) * 1000
            res.verify_ms += (t3 - t2) * 1000
            res.follow_rounds += 1
            res.round_nodes.append(len(tree.nodes))
            res.round_accepted.append(len(accepted))
            tokens.extend(accepted)
            if (accepted and accepted[-1] == self.eos) or len(tokens) >= cap_:
                return tokens
            cur = recovery

    def decode(self, fs: FrameState, candidates: list, datastore: Datastore | None = None,
               follow: str = "verify", new_coc: tuple | None = None) -> DecodeResult:
        """Decode one frame (respect.py:137-188 without the drafter).

        `candidates`: the previous CoCs (CocHistory.candidates(N)). follow="verify"
        runs follow-up verification from the datastore; follow="sequential"
        generates the rest one token per step. `new_coc` is added to the
        datastore's drive index inside the timed region.
        """
        datastore = datastore if datastore is not None else Datastore.empty(self.cfg.datastore_key_len)
        _sync(self.eng.device)
        t0 = time.perf_counter()
        insert_ms = 0.0
        if new_coc is not None:
            ti = time.perf_counter()
            datastore.add(new_coc)
            insert_ms = (time.perf_counter() - ti) * 1000
        acc, rec, nodes, ncand = self._initial(fs, candidates)
        tm = time.perf_counter()
        res = DecodeResult(tokens=[], target_runs=1, accepted_initial=len(acc), initial_nodes=nodes,
                           initial_candidates=ncand, datastore_insert_ms=insert_ms)
        if (acc and acc[-1] == self.eos) or len(acc) == fs.max_tokens:
            tokens = acc
        elif follow == "sequential":
            tail = sequential(self.eng, fs, rec, len(acc), self.eos, fs.max_tokens - len(acc), self.act)
            tokens = acc + tail
            res.target_runs = 1 + len(tail)
        else:
            tokens = self._follow(fs, acc, rec, datastore, res)
            res.target_runs = 1 + res.follow_rounds
        _sync(self.eng.device)
        t1 = time.perf_counter()
        res.tokens = [int(x) for x in tokens]
        res.initial_ms = (tm - t0) * 1000
        res.follow_ms = (t1 - tm) * 1000
        return res


def sequential(engine: VerifyEngine, fs: FrameState, token: int, base: int, eos: int, max_tokens: int,
               act: tuple = (0, 0)) -> list:
    """Token-by-token greedy decoding from `token` after `base` committed tokens, until EOS or
    `max_tokens`; returns the generated tokens including `token` (sequential.py:26-42)."""
    out = []
    one_parent, one_depth = np.array([-1], np.int32), np.array([0], np.int32)
    while len(out) < max_tokens:
        out.append(int(token))
        engine.step(np.array([token], np.int32), one_parent, one_depth, base + len(out) - 1, fs.prompt_len,
                    rope_delta=fs.rope_delta, act_off=act[0], act_size=act[1])
        if token == eos:
            break
        token = int(engine.fetch_ids(1)[0])
    return out
