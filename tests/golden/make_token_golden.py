"""Token-level golden fixture: accepted nodes and committed ids of the reference's
own verification rounds on a mid-size random Qwen3-VL text model.

Called by make_golden.py (``--only token``; the reference on sys.path). Runs on
CPU, in fp32 over bf16-valued weights, the reference's eager path, for each of
FRAMES seeded prompts:
  * HF Prefill of the prompt; the Prefill KV, rounded to bf16 values, is
    written into respect.decoding.kv_buffer.FixedKVBuffer (so the fixture's
    prefix KV is exactly representable in the bf16 engine that is compared);
  * the reference's token-by-token decoding of AR_LEN tokens from the Prefill's
    greedy pick, restated as 1-node respect.decoding.verify.verify_trie calls at
    base i (respect/decoding/sequential.py fixes device "cuda"; a 1-node trie at
    base i is the same forward);
  * round 1: a 48-node trie (the AR chain's first 24 tokens plus seeded sibling
    chains, topped up with seeded leaves) through verify_trie at base 0, then
    respect.decoding.acceptance.greedy_token (with an excluded vocabulary range)
    and walk, then respect.decoding.kv_buffer.compact;
  * round 2: a 32-node trie from the round-1 correction token at base
    len(accepted), the same way.
Stored per frame: the prompt, the bf16 prefix KV, the tries, both rounds'
per-node greedy ids and top-8 logits (values and indices), and the walks'
paths, tokens and correction tokens; frame 0's round-1 logits in full. The
weights are re-created by token_model(0) (seeded HF init) and checked against
per-tensor checksums.

Shims for transformers 5.5 as in make_model_golden.py: window-layer cache
positions from the harness, and the bf16 verify mask cast to fp32 for CPU SDPA.
"""
from __future__ import annotations

import numpy as np
import torch

TEXT = dict(hidden_size=512, intermediate_size=1536, num_hidden_layers=4, num_attention_heads=4,
            num_key_value_heads=2, head_dim=128, vocab_size=2048, rms_norm_eps=1e-6,
            rope_parameters=dict(rope_type="default", rope_theta=1e6, mrope_section=[24, 20, 20]))
VISION = dict(depth=1, hidden_size=64, intermediate_size=128, num_heads=2, out_hidden_size=512)
PL, CAP = 64, 96
FRAMES = 3
ACT_OFF, ACT_SIZE = 1500, 300        # the excluded (trajectory-token) vocabulary range
AR_LEN, R1_CHAIN, R1_NODES, R2_NODES = 36, 24, 48, 32


def token_model(seed=0):
    """The seeded random model, weights rounded to bf16 values (fp32 storage)."""
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration
    torch.manual_seed(seed)
    cfg = Qwen3VLConfig(text_config=TEXT, vision_config=VISION)
    cfg._attn_implementation = "sdpa"
    cfg.text_config._attn_implementation = "sdpa"
    m = Qwen3VLForConditionalGeneration(cfg).eval()
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    m.model.rope_deltas = torch.zeros(1, 1, dtype=torch.long)
    return m


def round1_seqs(chain, rng):
    """The AR chain's first R1_CHAIN tokens plus 3 seeded chains sharing a prefix with it."""
    from oracle.inputs import top_up
    from oracle.trie import build_trie as obuild
    base = tuple(chain[:R1_CHAIN])
    seqs = [base]
    for _ in range(3):
        share = int(rng.integers(1, R1_CHAIN))
        cand = base[:share] + tuple(int(t) for t in rng.integers(0, TEXT["vocab_size"], R1_CHAIN // 2))
        if len(obuild(seqs + [cand])[0]) <= R1_NODES:
            seqs.append(cand)
    return [tuple(s) for s in top_up(rng, seqs, R1_NODES, TEXT["vocab_size"])]


def round2_seqs(first, cont, rng):
    """Chains from the round-1 correction token: `cont` (the AR continuation, when the
    round committed an AR prefix) and seeded chains, topped up to R2_NODES."""
    from oracle.inputs import top_up
    V = TEXT["vocab_size"]
    seqs = [tuple([first] + list(cont))] if cont else []
    while len(seqs) < 3:
        seqs.append(tuple([first] + [int(t) for t in rng.integers(0, V, 6)]))
    return [tuple(s) for s in top_up(rng, seqs, R2_NODES, V)]


def generate(out_dir):
    import transformers.integrations.sdpa_attention as SA
    from respect.candidates.trie import build_trie
    from respect.decoding import kv_buffer
    from respect.decoding.acceptance import greedy_token, walk
    from respect.decoding.verify import verify_trie
    from respect.kernels import dispatch
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from make_model_golden import text_state, weight_checksum

    vlm = token_model(0)

    class Target:
        pass

    model = Target()
    model.vlm = vlm
    pos = {"p": None}

    def update(self, key_states, value_states, *args, **kwargs):   # shim 1
        self.keys.index_copy_(2, pos["p"], key_states)
        self.values.index_copy_(2, pos["p"], value_states)
        return self.keys, self.values

    kv_buffer.WindowLayer.update = update
    orig = dispatch.ORIG

    def sdpa_cast(module, query, key, value, attention_mask, *a, **kw):           # shim 2
        if attention_mask is not None and attention_mask.dtype not in (query.dtype, torch.bool):
            attention_mask = attention_mask.to(query.dtype)
        return orig(module, query, key, value, attention_mask, *a, **kw)

    SA.sdpa_attention_forward = sdpa_cast
    dispatch.ORIG = sdpa_cast
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa_cast

    V = TEXT["vocab_size"]
    arrays = {}
    for f in range(FRAMES):
        rng = np.random.default_rng(77 + f)
        prompt = torch.from_numpy(rng.integers(0, V, PL)).long()[None]
        with torch.no_grad():
            pf = vlm(input_ids=prompt, use_cache=True)
        first = int(greedy_token(pf.logits[0, -1:].float(), ACT_OFF, ACT_SIZE)[0])

        buf = kv_buffer.FixedKVBuffer(PL, (CAP,))
        buf.allocate(pf.past_key_values)
        buf.write_prefill(pf.past_key_values)
        with torch.no_grad():
            for t in buf.base_k + buf.base_v:
                t.copy_(t.to(torch.bfloat16).float())
        prefix = [(bk[0, :, :PL].clone(), bv[0, :, :PL].clone()) for bk, bv in zip(buf.base_k, buf.base_v)]

        def reset_prefix():
            for (k, v), bk, bv in zip(prefix, buf.base_k, buf.base_v):
                bk.zero_()
                bv.zero_()
                bk[0, :, :PL].copy_(k)
                bv[0, :, :PL].copy_(v)

        def run(tree, base):
            pos["p"] = torch.arange(PL + base, PL + base + len(tree.nodes))
            out = verify_trie(model, {"input_ids": prompt}, buf.window(CAP), tree, PL, base, CAP)
            return out.logits[0].float()

        # the reference's token-by-token decoding (1-node verify steps)
        chain = [first]
        for i in range(AR_LEN):
            lg = run(build_trie([(chain[-1],)]), i)
            chain.append(int(greedy_token(lg, ACT_OFF, ACT_SIZE)[0]))
        F = f"f{f}_"
        arrays[F + "ar_chain"] = np.array(chain, np.int64)

        reset_prefix()
        base, first_r, acc_all = 0, first, []
        for r, nodes in ((1, R1_NODES), (2, R2_NODES)):
            if r == 1:
                seqs = round1_seqs(chain, rng)
            else:
                cont = chain[base + 1:base + 12] if chain[base] == first_r and chain[:base] == acc_all else []
                seqs = round2_seqs(first_r, cont, rng)
            tree = build_trie(seqs)
            assert len(tree.nodes) == nodes, (r, len(tree.nodes))
            lg = run(tree, base)
            masked = lg.clone()
            masked[:, ACT_OFF:ACT_OFF + ACT_SIZE] = float("-inf")
            top8 = masked.topk(8, dim=-1)
            ids = greedy_token(lg, ACT_OFF, ACT_SIZE).tolist()
            path, acc, rec = walk(tree, first_r, 1 << 30, -1, lambda a, node: ids[node])
            kv_buffer.compact(buf.window(CAP), PL, base, path)
            p = f"{F}r{r}_"
            arrays[p + "parents"] = np.array([-1 if n.parent is None else n.parent for n in tree.nodes], np.int32)
            arrays[p + "tokens"] = np.array([n.token for n in tree.nodes], np.int32)
            arrays[p + "depths"] = np.array([n.depth for n in tree.nodes], np.int32)
            arrays[p + "meta"] = np.array([base, first_r, rec], np.int64)
            arrays[p + "greedy"] = np.array(ids, np.int64)
            arrays[p + "top8_val"] = top8.values.numpy().astype(np.float32)
            arrays[p + "top8_idx"] = top8.indices.numpy().astype(np.int32)
            arrays[p + "path"] = np.array(path, np.int64)
            arrays[p + "acc"] = np.array(acc, np.int64)
            if r == 1 and f == 0:
                arrays[p + "logits"] = lg.numpy().astype(np.float32)
            acc_all += list(acc)
            base += len(acc)
            first_r = rec
            print(f"token golden: frame {f} round {r}: {nodes} nodes, accepted {len(acc)}")
        for li, (k, v) in enumerate(prefix):
            arrays[f"{F}k{li}"] = k.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
            arrays[f"{F}v{li}"] = v.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        arrays[F + "prompt"] = prompt[0].numpy()
        arrays[F + "first"] = np.array([first], np.int64)
    arrays.update({f"wsum_{k}": weight_checksum(v) for k, v in text_state(vlm).items()})
    arrays["meta"] = np.array([PL, CAP, ACT_OFF, ACT_SIZE, FRAMES], np.int64)
    np.savez_compressed(out_dir / "token.npz", **arrays)
