"""Host side of the multi-stream frame replay (no GPU): the verification trie of
a round, the frame prompts, the prefill reuse rule, and the replay loop itself
driven over bigram stand-in engines."""
import numpy as np
import pytest

from respect_b200.decoding.replay import ReplayConfig, _Stream, round_trie


def test_round_trie_shape():
    rng = np.random.default_rng(0)
    rcfg = ReplayConfig(trie_nodes=256, chains=4, chain_len=48)
    t = round_trie(7, [(7, 1, 2, -1), (8, 1), (7, 1, 3)], rcfg, 1000, rng)
    assert len(t.nodes) == 256
    assert t.nodes[0].token == 7 and sum(1 for n in t.nodes if n.parent is None) == 1
    par, dep = t.parents(), t.depths()
    assert all(par[i] < i for i in range(256))
    assert all(dep[i] == (0 if par[i] < 0 else dep[par[i]] + 1) for i in range(256))
    # the out-of-vocabulary EOS ends the first chain; the chain from another root is dropped
    assert [n.token for n in t.nodes[:4]] == [7, 1, 2, 3]
    # siblings hold distinct tokens (one child per token)
    for n in t.nodes:
        assert len(n.children) == len(set(n.children))
    # the same seed gives the same trie
    t2 = round_trie(7, [(7, 1, 2, -1), (8, 1), (7, 1, 3)], rcfg, 1000, np.random.default_rng(0))
    assert t2.tokens().tolist() == t.tokens().tolist() and t2.parents().tolist() == par.tolist()


def test_round_trie_with_full_chains():
    rng = np.random.default_rng(1)
    rcfg = ReplayConfig(trie_nodes=256, chains=4, chain_len=48)
    cands = [(5,) + tuple(range(100 * k, 100 * k + 60)) for k in range(1, 7)]
    t = round_trie(5, cands, rcfg, 1000, rng)
    assert len(t.nodes) == 256
    # the first four candidates, cut to 48 tokens, are the first 1 + 4 * 47 nodes
    assert t.tokens()[:48].tolist() == list(cands[0][:48])
    assert 1 + 4 * 47 <= 256


def test_frame_prompts_share_the_configured_fraction():
    class _E:
        device = "cpu"

    rcfg = ReplayConfig(prompt_len=4096, shared_frac=0.9, seed=3)
    s = _Stream.__new__(_Stream)
    s.cfg, s.rng, s.prompt = rcfg, np.random.default_rng([3, 0]), None
    p0 = s.next_prompt(152064)
    assert p0.shape == (4096,) and p0.dtype == np.int32
    s.prompt = p0
    p1 = s.next_prompt(152064)
    changed = np.flatnonzero(p0 != p1)
    # one contiguous block of 10% (a random token may repeat the old one)
    assert len(changed) <= 410 and len(changed) > 380
    assert changed[-1] - changed[0] < 410


def test_prefill_reuse_start():
    from respect_b200.decoding.engine import prefill_start
    p = np.arange(1000)
    assert prefill_start(p, None, 256) == 0
    assert prefill_start(p, p, 256) == 768                # same prompt: only the last chunk
    q = p.copy(); q[0] = -1
    assert prefill_start(q, p, 256) == 0                  # first token changed
    q = p.copy(); q[300] = -1
    assert prefill_start(q, p, 256) == 256                # the chunk holding token 300 on
    q = p.copy(); q[255] = -1
    assert prefill_start(q, p, 256) == 0
    q = p.copy(); q[256] = -1
    assert prefill_start(q, p, 256) == 256
    assert prefill_start(p[:512], p, 256) == 256          # old prompt longer: last chunk of the new
    assert prefill_start(p, p[:600], 256) == 512          # old prompt shorter: from its last whole chunk
    assert prefill_start(p[:256], p, 256) == 0            # one chunk: it always runs
    assert prefill_start(p[:0], p, 256) == 0              # empty prompt: nothing to run
    assert prefill_start(p[:513], p[:513], 256) == 512


class _StubStream:
    def __init__(self, *a):
        pass

    def synchronize(self):
        pass


class _BigramReplayEngine:
    """The engine calls FrameReplay makes, over a bigram model (greedy pick after a
    token = (31 t + 7) mod V): prefill sets the pick after the prompt's last token."""
    device = "cpu"

    def __init__(self, rows, slots, vocab):
        self.max_rows, self.max_slots, self.vocab = rows, slots, vocab
        self.prompt = None
        self.prefilled = []

    def pick(self, t):
        return (int(t) * 31 + 7) % self.vocab

    def prefill(self, tokens, chunk=None, graph=True, reuse=None, stream=None):
        from respect_b200.decoding.engine import prefill_start
        toks = np.asarray(tokens)
        start = prefill_start(toks, reuse, chunk)
        self.prompt = toks
        self.last = np.array([self.pick(t) for t in toks[start:]])
        self.prefilled.append(len(toks) - start)
        return len(toks) - start

    def fetch_ids_async(self, q=None, stream=None):
        pass

    def ids_result(self):
        return self.last

    def step(self, ids, parents, depths, base, prompt_len, graph=True, stream=None, **kw):
        assert len(ids) <= self.max_rows and prompt_len + base + len(ids) <= self.max_slots
        self.ids, self.parents = np.asarray(ids).astype(int), np.asarray(parents).astype(int)

    def accept_async(self, first, cap, eos, n=None, stream=None):
        children = {}
        for i, p in enumerate(self.parents):
            children.setdefault(int(p), {})[int(self.ids[i])] = i
        path, acc, corr = [], [], first
        node = children.get(-1, {}).get(first)
        while node is not None and len(acc) < cap:
            path.append(node)
            acc.append(int(self.ids[node]))
            if acc[-1] == eos:
                break
            corr = self.pick(self.ids[node])
            node = children.get(node, {}).get(corr)
        self.rec = (path, acc, corr)

    def accept_result(self):
        return self.rec

    def close(self):
        pass


def test_frame_replay_host_loop(monkeypatch):
    """FrameReplay's loop over several streams: each frame commits exactly the model's
    continuation of its first token; the previous frames' CoCs and the datastore make
    later frames of an unchanged prompt finish in fewer rounds; prefill reuse follows
    prefill_start."""
    from types import SimpleNamespace

    from respect_b200.decoding import replay as rp
    from respect_b200.decoding.engine import prefill_start
    monkeypatch.setattr(rp.torch.cuda, "Stream", _StubStream)
    V = 97
    for shared in (1.0, 0.9):
        cfg = ReplayConfig(streams=3, prompt_len=50, shared_frac=shared, trie_nodes=16, chains=2, chain_len=6,
                           commit_tokens=12, prefill_chunk=16, seed=4)
        engines = [_BigramReplayEngine(16, cfg.max_slots(), V) for _ in range(cfg.streams)]
        rep = rp.FrameReplay(SimpleNamespace(cfg=SimpleNamespace(vocab=V)), cfg, engines=engines)
        st = rep.run(3, keep_records=True)
        assert st.frames == 9 and st.committed == 9 * 12 and len(st.records) == 9
        prev = {}
        for r in st.records:
            want = [r.first]
            while len(want) < 12:
                want.append((want[-1] * 31 + 7) % V)
            assert r.tokens == want and sum(r.accepted) == 12 and r.rounds == len(r.accepted)
            assert r.first == (int(r.prompt[-1]) * 31 + 7) % V
            old = prev.get(r.stream)
            assert r.prefill_tokens == len(r.prompt) - prefill_start(r.prompt, old, 16)
            if shared == 1.0 and old is not None:
                # the same prompt again: the last chunk only, and the first round takes a whole chain
                assert r.prefill_tokens == 50 - 48 and r.accepted[0] == 6 and r.rounds < 12
            prev[r.stream] = r.prompt
        rep.close()
    with pytest.raises(ValueError):
        rp.FrameReplay(SimpleNamespace(cfg=SimpleNamespace(vocab=V)), cfg,
                       engines=[_BigramReplayEngine(8, cfg.max_slots(), V)] * 3)
