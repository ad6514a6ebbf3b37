"""Model-level golden fixture: the reference's verify step on a tiny random Qwen3-VL.

Called by make_golden.py (which puts the reference on sys.path and sets
TRITON_INTERPRET=1). Runs, on CPU in fp32:
  * HF Prefill of a seeded prompt (default kernels),
  * respect.decoding.kv_buffer.FixedKVBuffer + respect.decoding.verify.verify_trie
    over a seeded trie, once on the default (eager SDPA) path and once inside
    respect.kernels.patch.dedicated_kernels (its Triton GEMM / RMSNorm /
    attention, interpreted),
and stores the inputs, both logits, the KV buffer of both layers and the
reference dispatch's kernel/fallback counters. The weights are not stored:
tiny_model(0) re-creates them (seeded HF init on CPU), and the fixture keeps a
per-tensor checksum that the tests assert before using them.

Two shims adapt the reference (written for transformers 4.57) to the image's
transformers 5.5: Cache.update no longer passes
cache_kwargs["cache_position"] (the window layer takes the positions from the
harness), and on CPU in fp32 eager SDPA needs the bf16 verify mask cast to the
query dtype.
"""
from __future__ import annotations

import numpy as np
import torch

TEXT = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
            num_key_value_heads=1, head_dim=128, vocab_size=1000, rms_norm_eps=1e-6,
            rope_parameters=dict(rope_type="default", rope_theta=1e6, mrope_section=[24, 20, 20]))
VISION = dict(depth=1, hidden_size=64, intermediate_size=128, num_heads=2, out_hidden_size=256)
PL, CAP = 40, 64


def tiny_model(seed=0):
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration
    torch.manual_seed(seed)
    cfg = Qwen3VLConfig(text_config=TEXT, vision_config=VISION)
    cfg._attn_implementation = "sdpa"
    cfg.text_config._attn_implementation = "sdpa"
    m = Qwen3VLForConditionalGeneration(cfg).eval()
    m.model.rope_deltas = torch.zeros(1, 1, dtype=torch.long)
    return m


def text_state(vlm):
    """The text model's weights as numpy fp32 (name -> array)."""
    lm = vlm.model.language_model
    out = {"embed": vlm.model.language_model.embed_tokens.weight, "lm_head": vlm.lm_head.weight,
           "final_norm": lm.norm.weight}
    for i, layer in enumerate(lm.layers):
        a, mlp = layer.self_attn, layer.mlp
        for n, t in (("q", a.q_proj.weight), ("k", a.k_proj.weight), ("v", a.v_proj.weight), ("o", a.o_proj.weight),
                     ("qn", a.q_norm.weight), ("kn", a.k_norm.weight), ("g", mlp.gate_proj.weight),
                     ("u", mlp.up_proj.weight), ("d", mlp.down_proj.weight), ("in", layer.input_layernorm.weight),
                     ("post", layer.post_attention_layernorm.weight)):
            out[f"l{i}_{n}"] = t
    return {k: v.detach().float().numpy() for k, v in out.items()}


def weight_checksum(a):
    """float64 sum, sum of squares and the first/last elements of one weight."""
    f = np.asarray(a, np.float64).ravel()
    return np.array([f.sum(), (f * f).sum(), f[0], f[-1]])


def generate(out_dir):
    import transformers.integrations.sdpa_attention as SA
    from respect.candidates.trie import build_trie
    from respect.decoding import kv_buffer
    from respect.decoding.verify import verify_trie
    from respect.kernels import dispatch
    from respect.kernels.patch import dedicated_kernels
    from oracle.inputs import chain_seqs, top_up

    vlm = tiny_model(0)

    class Target:
        pass

    model = Target()
    model.vlm = vlm
    rng = np.random.default_rng(21)
    prompt = torch.from_numpy(rng.integers(0, 1000, PL)).long()[None]
    seqs = top_up(rng, chain_seqs(rng, 3, 8, 1000), 20, 1000)
    tree = build_trie([tuple(s) for s in seqs])
    q = len(tree.nodes)

    # shim 1: the window layer writes at the positions the harness sets
    pos = {"p": None}

    def update(self, key_states, value_states, *args, **kwargs):
        self.keys.index_copy_(2, pos["p"], key_states)
        self.values.index_copy_(2, pos["p"], value_states)
        return self.keys, self.values

    kv_buffer.WindowLayer.update = update
    # shim 2: eager SDPA on CPU fp32 wants the additive mask in the query dtype
    orig = dispatch.ORIG

    def sdpa_cast(module, query, key, value, attention_mask, *a, **kw):
        if attention_mask is not None and attention_mask.dtype != query.dtype and attention_mask.dtype != torch.bool:
            attention_mask = attention_mask.to(query.dtype)
        return orig(module, query, key, value, attention_mask, *a, **kw)

    SA.sdpa_attention_forward = sdpa_cast
    dispatch.ORIG = sdpa_cast
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa_cast

    with torch.no_grad():
        pf = vlm(input_ids=prompt, use_cache=True)
    arrays = {}
    for name, ctx in (("eager", None), ("dedicated", True)):
        buf = kv_buffer.FixedKVBuffer(PL, (CAP,))
        buf.allocate(pf.past_key_values)
        buf.write_prefill(pf.past_key_values)
        cache = buf.window(CAP)
        pos["p"] = torch.arange(PL, PL + q)
        if ctx:
            with dedicated_kernels(model, PL):
                out = verify_trie(model, {"input_ids": prompt}, cache, tree, PL, 0, CAP)
        else:
            out = verify_trie(model, {"input_ids": prompt}, cache, tree, PL, 0, CAP)
        arrays[f"logits_{name}"] = out.logits[0].float().numpy()
        for li in range(len(buf.base_k)):
            arrays[f"k{li}_{name}"] = buf.base_k[li][0, :, :PL + q].numpy()
            arrays[f"v{li}_{name}"] = buf.base_v[li][0, :, :PL + q].numpy()
        arrays[f"stats_{name}"] = np.array([dispatch.STATS["kernel"], dispatch.STATS["fallback"]])
        dispatch.STATS.update(kernel=0, fallback=0)
    arrays.update({f"wsum_{k}": weight_checksum(v) for k, v in text_state(vlm).items()})
    arrays["prompt"] = prompt[0].numpy()
    arrays["trie_parents"] = np.array([-1 if n.parent is None else n.parent for n in tree.nodes], np.int32)
    arrays["trie_tokens"] = np.array([n.token for n in tree.nodes], np.int64)
    arrays["trie_depths"] = np.array([n.depth for n in tree.nodes], np.int32)
    arrays["seqs_flat"] = np.array([t for s in tree.seqs for t in s], np.int64)
    arrays["seqs_len"] = np.array([len(s) for s in tree.seqs], np.int64)
    arrays["meta"] = np.array([PL, CAP])
    np.savez_compressed(out_dir / "model.npz", **arrays)
