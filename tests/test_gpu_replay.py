"""Multi-stream frame replay reproduces token-by-token decoding on every stream.

Several frame streams run concurrently on one GPU (own KV buffers and CUDA
streams, shared weights), with Prefill reusing the unchanged chunks of the
previous frame's prompt. Every frame of every stream must equal a fresh engine
that prefills the same prompt from scratch and then decodes one token per step
(respect/decoding/sequential.py:26-42): same first token, same committed
tokens; and for each stream's last frame, the same KV slots bit for bit.
"""
import pytest
import torch

from respect_b200.decoding.engine import DecoderConfig, DecoderWeights, VerifyEngine
from respect_b200.decoding.replay import FrameReplay, ReplayConfig
from respect_b200.decoding.respect import FrameState, sequential

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def model():
    cfg = DecoderConfig.tiny(2)
    return cfg, DecoderWeights.random(cfg, DEV, seed=3, std=0.02)


def _check(w, rcfg, rep, stats):
    ref = VerifyEngine(w, max_rows=max(rcfg.trie_nodes, rcfg.prefill_chunk), max_slots=rcfg.max_slots())
    pl, n = rcfg.prompt_len, rcfg.commit_tokens
    last = {}
    for r in stats.records:
        last[r.stream] = r
    try:
        for r in stats.records:
            ref.prefill(r.prompt, chunk=rcfg.prefill_chunk)
            first = int(ref.fetch_ids()[-1])
            assert first == r.first, (r.stream, r.frame)
            toks = sequential(ref, FrameState(pl, first, n), first, 0, rcfg.eos, n)
            assert toks == r.tokens, (r.stream, r.frame, r.accepted)
            if last[r.stream] is r:
                eng = rep.streams[r.stream].eng
                for l in range(w.cfg.n_layers):
                    assert torch.equal(eng.kc[l][:, :pl + n], ref.kc[l][:, :pl + n]), (r.stream, l)
                    assert torch.equal(eng.vc[l][:, :pl + n], ref.vc[l][:, :pl + n]), (r.stream, l)
    finally:
        ref.close()


@pytest.mark.parametrize("shared,one_cuda_stream", [(0.9, False), (1.0, True)])
def test_replay_streams_equal_sequential(model, shared, one_cuda_stream):
    cfg, w = model
    rcfg = ReplayConfig(streams=3, prompt_len=200, shared_frac=shared, trie_nodes=64, chains=4, chain_len=12,
                        commit_tokens=20, prefill_chunk=64, seed=7, shared_cuda_stream=one_cuda_stream)
    rep = FrameReplay(w, rcfg)
    try:
        stats = rep.run(3, keep_records=True)
        assert stats.frames == 9 and len(stats.records) == 9
        assert all(len(r.tokens) == rcfg.commit_tokens for r in stats.records)
        later = [r for r in stats.records if r.frame > 0]
        if shared == 1.0:
            # the same prompt again: only the last chunk is recomputed, and the previous
            # CoC holds the whole continuation, so the first round accepts a full chain
            assert all(r.prefill_tokens == 200 - 192 for r in later)
            assert all(r.accepted[0] >= rcfg.chain_len for r in later)
            assert all(r.rounds < rcfg.commit_tokens for r in later)
        else:
            assert all(r.prefill_tokens <= 200 for r in later)
        _check(w, rcfg, rep, stats)
    finally:
        rep.close()

