"""Parity of the native engine with outside references, at full size and at the
token level (BASELINE config 3 and the north-star parity bar).

* Token level: the engine driven through the reference's own verification
  rounds (tests/golden/token.npz, the reference's eager path on a 4-layer random
  Qwen3-VL text model): logits within 2e-2, every node's greedy id and every
  acceptance walk equal to the reference's except at reported near-ties
  (tests/token_parity.py).
* Full size: the config-3 verify step (hidden 3584, 28 / 4 heads of 128, FFN
  18944, vocab 152,064, prefix 3,000, 128-node trie) against an independent
  fp32 restatement of the reference's math on the same GPU over the same bf16
  weights and the same prefix KV (oracle/torch_model.py): logits, node K / V and
  greedy ids, for the first two layers plus the final norm and lm_head, and for
  the whole 28-layer model.
"""
import numpy as np
import pytest
import torch

from oracle import torch_model as tm
from oracle.inputs import chain_seqs, top_up
from respect_b200.candidates.trie import build_trie
from respect_b200.decoding.engine import DecoderConfig, DecoderWeights, VerifyEngine
from tests import token_parity as tp

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


def test_engine_token_parity_with_reference():
    from respect_b200.kernels.gemm import interleave_gate_up
    z = tp.load()
    PL, CAP = int(z["meta"][0]), int(z["meta"][1])
    st = tp.model_state(z)
    cfg = DecoderConfig(512, 4, 4, 2, 128, 1536, 2048)

    def t(name):
        return torch.from_numpy(st[name]).to(DEV, torch.bfloat16)

    layers = [dict(wqkv=torch.cat([t(f"l{i}_q"), t(f"l{i}_k"), t(f"l{i}_v")]), wo=t(f"l{i}_o"),
                   wgu=interleave_gate_up(t(f"l{i}_g"), t(f"l{i}_u")).contiguous(), wd=t(f"l{i}_d"),
                   in_norm=t(f"l{i}_in"), post_norm=t(f"l{i}_post"), q_norm=t(f"l{i}_qn"), k_norm=t(f"l{i}_kn"))
              for i in range(4)]
    w = DecoderWeights(cfg, t("embed"), t("lm_head"), t("final_norm"), layers)
    eng = VerifyEngine(w, max_rows=64, max_slots=PL + CAP)
    try:
        def reset_frame(f):
            for li, (k, v) in enumerate(tp.prefix_kv(z, f, 4)):
                eng.kc[li].zero_()
                eng.vc[li].zero_()
                eng.kc[li][:, :PL] = torch.from_numpy(k).to(DEV, torch.bfloat16)
                eng.vc[li][:, :PL] = torch.from_numpy(v).to(DEV, torch.bfloat16)

        def run_round(tokens, parents, depths, base, off, size):
            eng.step(np.asarray(tokens, np.int32), np.asarray(parents, np.int32), np.asarray(depths, np.int32),
                     base, PL, act_off=off, act_size=size)
            q = len(tokens)
            return eng.logits(q).cpu().numpy(), eng.next_ids(q).cpu().numpy()

        def compact(path, base):
            eng.compact(path, PL, base)

        rep = tp.check_rounds(z, run_round, reset_frame, compact)
    finally:
        eng.close()
    print("engine vs reference:", {k: v for k, v in rep.items() if k != "ties"}, "tie events:", rep["ties"])
    assert rep["nodes"] == 3 * (48 + 32)
    assert rep["committed_equal"] >= 0.5 * tp.committed_total(z)


def _full_size_case(n_layers):
    cfg = DecoderConfig(3584, n_layers, 28, 4, 128, 18944, 152064)
    w = DecoderWeights.random(cfg, DEV, seed=0)
    P, NODES = 3000, 128
    eng = VerifyEngine(w, max_rows=NODES, max_slots=P + 256)
    rng = np.random.default_rng(9)
    eng.prefill(rng.integers(0, cfg.vocab, P))
    tree = build_trie(top_up(rng, chain_seqs(rng, 4, 32, cfg.vocab), NODES, cfg.vocab))
    assert len(tree.nodes) == NODES
    kc = [k.clone() for k in eng.kc]       # the engine's prefix KV, for the restatement
    vc = [v.clone() for v in eng.vc]
    eng.step(tree.tokens().astype(np.int32), tree.parents(), tree.depths(), 0, P)
    got = eng.logits(NODES).clone()
    ids = eng.next_ids(NODES).clone()
    ref = tm.verify_step(tm.weights_of(w), tm.cfg_of(cfg), tree.tokens(), tree.parents(), tree.depths(), P, 0,
                         kc, vc, mode="fp32")
    err = (got - ref).abs().max().item()
    kerr = max(max((eng.kc[li][:, P:P + NODES].float() - kc[li][:, P:P + NODES].float()).abs().max().item(),
                   (eng.vc[li][:, P:P + NODES].float() - vc[li][:, P:P + NODES].float()).abs().max().item())
               for li in range(n_layers))
    top2 = ref.topk(2, dim=-1).values
    margin = (top2[:, 0] - top2[:, 1]).cpu().numpy()
    flips = np.flatnonzero(ids.cpu().numpy() != ref.argmax(-1).cpu().numpy())
    eng.close()
    print(f"config-3 engine, {n_layers} layers, vs fp32 restatement: logits max-abs {err:.3e} "
          f"(|logits| max {ref.abs().max().item():.2f}), node K/V max-abs {kerr:.3e}, "
          f"greedy flips {[(int(n), float(margin[n])) for n in flips]}")
    return err, kerr, flips, margin


def test_config3_two_layers_vs_fp32_restatement():
    """Every config-3 kernel at full size (q|k|v, attention over 3,000 + 128 keys, o,
    gate|up + SiLU*mul, down, norms, lm_head over 152,064 rows) through two layers."""
    err, kerr, flips, margin = _full_size_case(2)
    assert err <= TOL, err
    assert kerr <= 0.05, kerr            # a bf16 ulp of the largest K / V values
    assert all(margin[n] < TOL for n in flips)


def test_config3_28_layers_vs_fp32_restatement():
    """The whole config-3 model (the step bench.py times) against the restatement."""
    err, kerr, flips, margin = _full_size_case(28)
    assert err <= TOL, err
    assert all(margin[n] < TOL for n in flips)
