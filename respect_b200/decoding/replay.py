"""Multi-stream frame replay on the native verify engine.

A drive is a sequence of frames. Each frame is a prompt (Prefill) followed by
verification rounds until `commit_tokens` tokens are committed or EOS: the
per-frame loop of respect/decoding/respect.py:137-188, with the previous
frames' CoCs as candidates (respect/candidates/history.py:1-50) and the drive's
datastore (respect/candidates/datastore.py) for the follow-up rounds.

Several independent drives (frame streams) share one GPU. Each stream has
its own KV buffer and workspace (`VerifyEngine(share_weights=...)`: the model
weights are held once) and its own CUDA stream. One host thread keeps all of
them in flight: while the device runs other streams' steps, the host reads
stream a's acceptance record (`accept_async` / `accept_result`) and builds a's
next trie. Across GPUs the streams are replicas: one process per GPU, no
collective.

Workload (the frame-replay measurement configuration):
  * frame 0 of a stream is `prompt_len` seeded random tokens; each later frame
    keeps `shared_frac` of the previous prompt and replaces one contiguous block
    (at a seeded offset) with seeded random tokens, as a new camera image
    replaces the image tokens between an unchanged system prompt and question;
  * Prefill runs the prompt in `prefill_chunk`-token chunks and keeps the KV of
    the whole chunks before the first changed token (exact:
    `VerifyEngine.prefill(reuse=...)`); the last row's greedy pick is the
    frame's first token;
  * every verification round runs a trie of exactly `trie_nodes` nodes: up to
    `chains` candidate chains of `chain_len` tokens from the root (the
    first-token-filtered CoCs of the last `chains` frames in the first round;
    the datastore's continuations of the committed tokens after it), seeded
    random chains when there are fewer, and seeded continuation nodes under
    seeded nodes until the trie holds `trie_nodes` nodes;
  * acceptance and KV compaction run on the device; the frame ends at
    `commit_tokens` committed tokens or EOS, and its tokens become the newest
    CoC of the stream's history and datastore.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from respect_b200.candidates.datastore import Datastore
from respect_b200.candidates.history import CocHistory, first_token_filter
from respect_b200.candidates.trie import Node, Trie, build_trie
from respect_b200.decoding.engine import DecoderWeights, VerifyEngine


@dataclass(frozen=True)
class ReplayConfig:
    streams: int = 16
    prompt_len: int = 4096
    shared_frac: float = 0.9
    trie_nodes: int = 256
    chains: int = 4
    chain_len: int = 48
    commit_tokens: int = 80
    prefill_chunk: int = 256
    reuse_prefix: bool = True
    eos: int = -1
    datastore_key_len: int = 2
    seed: int = 0
    shared_cuda_stream: bool = False  # every frame stream's work on one CUDA stream, in host order

    def max_slots(self) -> int:
        # the last round writes its nodes after at most commit_tokens - 1 committed tokens
        return self.prompt_len + self.commit_tokens + self.trie_nodes


@dataclass
class FrameRecord:
    stream: int
    frame: int
    first: int
    tokens: list
    rounds: int
    accepted: list
    prefill_tokens: int
    prompt: np.ndarray | None = None


@dataclass
class ReplayStats:
    frames: int = 0
    rounds: int = 0
    prefill_steps: int = 0
    prefill_tokens: int = 0
    committed: int = 0
    records: list = field(default_factory=list)

    def tokens_per_round(self) -> float:
        return self.committed / max(self.rounds, 1)


def top_up(tree: Trie, n_nodes: int, vocab: int, rng: np.random.Generator) -> Trie:
    """Add seeded continuation nodes (a random token under a random existing node,
    distinct from that node's children) until the trie has `n_nodes` nodes."""
    while len(tree.nodes) < n_nodes:
        par = int(rng.integers(0, len(tree.nodes)))
        tok = int(rng.integers(0, vocab))
        node = tree.nodes[par]
        if tok in node.children:
            continue
        node.children[tok] = len(tree.nodes)
        tree.nodes.append(Node(tok, par, node.depth + 1))
    return tree


def round_trie(root: int, cands: list, cfg: ReplayConfig, vocab: int, rng: np.random.Generator) -> Trie:
    """The verification trie of one round: candidate chains from `root`, cut to
    chain_len, at most cfg.chains of them, seeded chains in place of missing ones,
    seeded continuation nodes up to cfg.trie_nodes."""
    chains: list = []
    for c in cands:
        c = [int(t) for t in c[:cfg.chain_len]]
        bad = [i for i, t in enumerate(c) if not 0 <= t < vocab]  # EOS outside the vocabulary ends a chain
        c = tuple(c[:bad[0]] if bad else c)
        if c and c[0] == root and c not in chains:
            chains.append(c)
        if len(chains) == cfg.chains:
            break
    while len(chains) < cfg.chains:
        chains.append((root,) + tuple(int(t) for t in rng.integers(0, vocab, cfg.chain_len - 1)))
    tree = build_trie(chains)
    if len(tree.nodes) > cfg.trie_nodes:
        raise ValueError(f"{cfg.chains} chains of {cfg.chain_len} exceed {cfg.trie_nodes} nodes")
    return top_up(tree, cfg.trie_nodes, vocab, rng)


class _Stream:
    def __init__(self, idx: int, eng: VerifyEngine, cfg: ReplayConfig, cuda=None):
        self.idx, self.eng, self.cfg = idx, eng, cfg
        self.cuda = cuda if cuda is not None else torch.cuda.Stream(eng.device)
        self.rng = np.random.default_rng([cfg.seed, idx])
        self.history = CocHistory(cfg.eos)
        self.store = Datastore.empty(cfg.datastore_key_len)
        self.prompt: np.ndarray | None = None
        self.frame = -1
        self.frames_left = 0
        self.pending: str | None = None  # "first" | "round"
        self.first = 0
        self.cur = 0
        self.committed: list = []
        self.accepted: list = []
        self.prefill_tokens = 0

    def next_prompt(self, vocab: int) -> np.ndarray:
        cfg, rng = self.cfg, self.rng
        if self.prompt is None:
            return rng.integers(0, vocab, cfg.prompt_len).astype(np.int32)
        p = self.prompt.copy()
        n_edit = int(round((1.0 - cfg.shared_frac) * cfg.prompt_len))
        if n_edit > 0:
            off = int(rng.integers(0, cfg.prompt_len - n_edit + 1))
            p[off:off + n_edit] = rng.integers(0, vocab, n_edit)
        return p


class FrameReplay:
    """`streams` frame streams on one device, one engine each, weights shared."""

    def __init__(self, weights: DecoderWeights, cfg: ReplayConfig = ReplayConfig(), graph: bool = True,
                 engines: list | None = None):
        """`engines`: one engine per stream, built by the caller (with at least
        max(trie_nodes, prefill_chunk) rows and cfg.max_slots() slots); by default one
        VerifyEngine per stream on shared packed weights."""
        self.cfg = cfg
        self.w = weights
        self.graph = graph
        self.vocab = weights.cfg.vocab
        rows = max(cfg.trie_nodes, cfg.prefill_chunk)
        if engines is None:
            engines = []
            for i in range(cfg.streams):
                engines.append(VerifyEngine(weights, max_rows=rows, max_slots=cfg.max_slots(),
                                            share_weights=engines[0] if engines else None))
        elif len(engines) != cfg.streams:
            raise ValueError(f"{len(engines)} engines for {cfg.streams} streams")
        for e in engines:
            if e.max_rows < rows or e.max_slots < cfg.max_slots():
                raise ValueError(f"engine of {e.max_rows} rows / {e.max_slots} slots is too small for "
                                 f"{rows} rows / {cfg.max_slots()} slots")
        shared = torch.cuda.Stream(engines[0].device) if cfg.shared_cuda_stream else None
        self.streams = [_Stream(i, e, cfg, shared) for i, e in enumerate(engines)]
        self.stats = ReplayStats()
        self.keep_records = False

    # ------------------------------------------------------------ per-stream steps
    def _start_frame(self, s: _Stream) -> None:
        cfg = self.cfg
        prompt = s.next_prompt(self.vocab)
        reuse = s.prompt if (cfg.reuse_prefix and s.prompt is not None) else None
        s.prefill_tokens = s.eng.prefill(prompt, chunk=cfg.prefill_chunk, graph=self.graph, reuse=reuse,
                                         stream=s.cuda)
        self.stats.prefill_steps += -(-s.prefill_tokens // cfg.prefill_chunk)
        self.stats.prefill_tokens += s.prefill_tokens
        s.prompt = prompt
        s.frame += 1
        s.frames_left -= 1
        s.eng.fetch_ids_async(stream=s.cuda)
        s.pending = "first"

    def _launch_round(self, s: _Stream) -> None:
        cfg = self.cfg
        base = len(s.committed)
        if base == 0:
            cands = first_token_filter(s.history.candidates(cfg.chains), s.cur)
        else:
            cands = [(s.cur,) + tuple(c) for c in s.store.lookup(s.committed + [s.cur])]
        tree = round_trie(s.cur, cands, cfg, self.vocab, s.rng)
        s.eng.step(tree.tokens().astype(np.int32), tree.parents(), tree.depths(), base, cfg.prompt_len,
                   graph=self.graph, stream=s.cuda)
        s.eng.accept_async(s.cur, cfg.commit_tokens - base, cfg.eos, n=len(tree.nodes), stream=s.cuda)
        s.pending = "round"

    def _finish_frame(self, s: _Stream) -> None:
        toks = [int(t) for t in s.committed]
        s.history.append(s.frame, toks)
        s.store.add(tuple(toks))
        self.stats.frames += 1
        self.stats.committed += len(toks)
        if self.keep_records:
            self.stats.records.append(FrameRecord(s.idx, s.frame, s.first, toks, len(s.accepted), list(s.accepted),
                                                  s.prefill_tokens, s.prompt.copy()))

    def _advance(self, s: _Stream) -> bool:
        """Consume s's finished piece and enqueue the next; False once s has no frames left."""
        if s.pending == "first":
            s.first = s.cur = int(s.eng.ids_result()[-1])
            s.committed, s.accepted = [], []
            self._launch_round(s)
            return True
        path, toks, corr = s.eng.accept_result()
        self.stats.rounds += 1
        s.committed.extend(int(t) for t in toks)
        s.accepted.append(len(toks))
        done = (toks and toks[-1] == self.cfg.eos) or len(s.committed) >= self.cfg.commit_tokens
        if not done:
            s.cur = corr
            self._launch_round(s)
            return True
        self._finish_frame(s)
        if s.frames_left > 0:
            self._start_frame(s)
            return True
        s.pending = None
        return False

    # ------------------------------------------------------------ driver
    def run(self, frames_per_stream: int, keep_records: bool = False) -> ReplayStats:
        """Replay `frames_per_stream` frames on every stream (continuing each drive);
        returns the counts of this call. Returns with every stream's work finished."""
        self.keep_records = keep_records
        self.stats = ReplayStats()
        if frames_per_stream <= 0:
            return self.stats
        for s in self.streams:
            s.frames_left = frames_per_stream
            self._start_frame(s)
        active = list(self.streams)
        while active:
            active = [s for s in active if self._advance(s)]
        for s in self.streams:
            s.cuda.synchronize()
        return self.stats

    def timed_run(self, frames_per_stream: int) -> tuple[ReplayStats, float]:
        """run() bracketed by CUDA events on the device (all streams drained on both sides): (stats, ms)."""
        dev = self.streams[0].eng.device
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        st = self.run(frames_per_stream)
        t1.record()
        torch.cuda.synchronize(dev)
        return st, t0.elapsed_time(t1)

    def close(self) -> None:
        for s in self.streams:
            s.eng.close()
