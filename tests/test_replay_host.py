"""Host side of the multi-stream frame replay: the verification trie of a round
and the frame prompts (no GPU)."""
import numpy as np

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
