"""Generate the golden fixtures in this folder by running the REFERENCE's own code.

    python tests/golden/make_golden.py --ref <path to a soonhong99/respect checkout>

What runs (all on CPU, in the build container where the reference is importable):
  * respect.candidates.trie.build_trie / trie_ancestry and
    respect.decoding.acceptance.walk on seeded candidate sets      -> trie.json
  * respect.decoding.verify.verify_trie with a stub model that records the
    ids / cache positions / rotary positions / 4-D mask it would feed  -> verify_mask.npz
  * respect.kernels.attention.fused_attn_hyb, .gemm.linear and
    .rmsnorm.rmsnorm, Triton kernels under TRITON_INTERPRET=1, fp32    -> kernels.npz
  * respect.kernels.dispatch.unified_forward (padding, node mask,
    causal mask, padding-row trick)                                    -> kernels.npz
  * PyTorch eager RoPE (q*cos + rotate_half(q)*sin) and silu(g)*u in
    bf16: the outputs respect/system/fused.py reproduces bitwise      -> kernels.npz
  * respect.candidates.datastore.Datastore lookups (static / drive /
    added / drive-only indexes, key lengths 1-3) and
    respect.candidates.history.CocHistory / first_token_filter on seeded
    sentences                                                          -> candidates.json
  * a 2-layer random-init Qwen3-VL text model verified through
    respect.decoding.verify.verify_trie with and without
    respect.kernels.patch.dedicated_kernels, fp32                       -> model.npz
  * two verification rounds (verify_trie, greedy_token, walk, compact) of
    the reference's eager path on a 4-layer random Qwen3-VL text model, and
    its token-by-token decoding, fp32, for 3 prompts (``--only token``) -> token.npz

Inputs come from oracle.inputs (seeded numpy); fixtures store outputs plus a
checksum of the inputs, so the tests regenerate the inputs and compare.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle.inputs import attention_case, chain_seqs, checksum, config1_trie, top_up  # noqa: E402


def trie_cases():
    eos = 99
    cases = [
        dict(name="shared_prefix", seqs=[(1, 2, 3, eos), (1, 2, 4, eos), (1, 2, 3, eos)]),
        dict(name="parent_before_child", seqs=[(1, 2, 3), (1, 5)]),
        dict(name="single_eos", seqs=[(1, eos)]),
        dict(name="empty_and_dupes", seqs=[(), (7,), (7,), (7, 8), ()]),
        dict(name="config1", seqs=[tuple(s) for s in config1_trie(0)]),
    ]
    rng = np.random.default_rng(3)
    for i in range(4):
        seqs = chain_seqs(rng, 4, 32, 50)
        cases.append(dict(name=f"chains32_{i}", seqs=[tuple(s) for s in top_up(rng, seqs, 128, 50)]))
    return cases


def gen_trie(out):
    from respect.candidates.trie import build_trie, trie_ancestry
    from respect.decoding.acceptance import walk
    res = []
    rng = np.random.default_rng(11)
    for c in trie_cases():
        t = build_trie(c["seqs"])
        anc = trie_ancestry(t)
        nodes = [[n.token, -1 if n.parent is None else n.parent, n.depth] for n in t.nodes]
        walks = []
        if t.nodes:
            for w in range(3):
                # target choice after each node: a child token with prob 0.8, else a fresh token
                target = {}
                for i, n in enumerate(t.nodes):
                    kids = list(n.children.keys())
                    if kids and rng.random() < 0.8:
                        target[i] = int(kids[int(rng.integers(0, len(kids)))])
                    else:
                        target[i] = int(rng.integers(1000, 2000))
                first = int(list(t.roots.keys())[int(rng.integers(0, len(t.roots)))])
                cap = [128, 5, 2][w]
                path, acc, rec = walk(t, first, cap, 99, lambda a, ch, tg=target: tg[ch])
                walks.append(dict(first=first, cap=cap, eos=99, target={str(k): v for k, v in target.items()},
                                  path=path, acc=acc, rec=int(rec)))
        res.append(dict(name=c["name"], seqs=[list(s) for s in c["seqs"]], nodes=nodes,
                        roots=[[int(k), int(v)] for k, v in t.roots.items()],
                        unique=[list(s) for s in t.seqs],
                        ancestry=[np.flatnonzero(anc[i]).tolist() for i in range(len(t.nodes))],
                        walks=walks))
    (out / "trie.json").write_text(json.dumps(res))


class _Capture:
    """Stub target: verify_trie only needs model.vlm(...) and model.vlm.model.rope_deltas."""

    def __init__(self, rope_delta):
        class _Inner:
            pass
        self.vlm = self
        self.model = _Inner()
        self.model.rope_deltas = torch.tensor([[rope_delta]])
        self.kw = None

    def __call__(self, **kw):
        self.kw = kw
        return None


def gen_verify_mask(out):
    from respect.candidates.trie import build_trie
    from respect.decoding.verify import verify_trie
    arrays = {}
    for i, (seqs, PL, base, cap, delta) in enumerate([
        ([(5, 6, 7), (5, 6, 8, 9), (5, 10)], 20, 0, 16, 0),
        ([tuple(s) for s in config1_trie(0)], 64, 7, 192, -3),
    ]):
        t = build_trie(seqs)
        stub = _Capture(delta)
        prepared = {"input_ids": torch.zeros(1, 1, dtype=torch.long)}
        verify_trie(stub, prepared, None, t, PL, base, cap)
        kw = stub.kw
        arrays[f"c{i}_ids"] = kw["input_ids"].numpy()
        arrays[f"c{i}_cache_position"] = kw["cache_position"].numpy()
        arrays[f"c{i}_position_ids"] = kw["position_ids"].numpy()
        arrays[f"c{i}_mask_bits"] = kw["attention_mask"].view(torch.int16).numpy().view(np.uint16)
        arrays[f"c{i}_meta"] = np.array([PL, base, cap, delta])
        arrays[f"c{i}_parents"] = np.array([-1 if n.parent is None else n.parent for n in t.nodes], np.int32)
        arrays[f"c{i}_depths"] = np.array([n.depth for n in t.nodes], np.int32)
        arrays[f"c{i}_tokens"] = np.array([n.token for n in t.nodes], np.int64)
    np.savez_compressed(out / "verify_mask.npz", **arrays)


def gen_kernels(out):
    from respect.kernels import dispatch
    from respect.kernels.attention import fused_attn_hyb
    from respect.kernels.gemm import linear
    from respect.kernels.rmsnorm import rmsnorm
    arrays = {}

    # Config 1: single-layer trie attention, fp32, through the kernel as dispatch pads it.
    c = attention_case(0)
    M = c["q"].shape[1]
    MP = ((M + 63) // 64) * 64
    qp = np.zeros((c["q"].shape[0], MP, 128), np.float32)
    qp[:, :M] = c["q"]
    msk = np.zeros((MP, c["msk"].shape[1]), bool)
    msk[:M] = c["msk"]
    msk[M:, 0] = True
    o = fused_attn_hyb(torch.from_numpy(qp), torch.from_numpy(c["kp"]), torch.from_numpy(c["vp"]),
                       torch.from_numpy(c["kn"]), torch.from_numpy(c["vn"]), torch.from_numpy(msk),
                       BM=64, BN=128, BNB=16, num_warps=4, num_stages=1)
    arrays["attn_c1_out"] = o[:, :M].numpy()
    arrays["attn_c1_checksum"] = np.array(checksum(*[c[k] for k in ("q", "kp", "vp", "kn", "vn", "msk")]))

    # dispatch.unified_forward: small case with a 4-D additive mask, and the causal case.
    rng = np.random.default_rng(5)
    H, HK, D, PL, cap = 4, 2, 128, 70, 40
    key = torch.from_numpy(rng.standard_normal((1, HK, PL + cap, D), dtype=np.float32))
    val = torch.from_numpy(rng.standard_normal((1, HK, PL + cap, D), dtype=np.float32))
    dispatch.install(PL)
    try:
        # trie of 5 nodes after 3 committed tokens, inside a window of PL + cap keys
        parents = [-1, 0, 1, 0, 3]
        from oracle.trie import ancestry
        anc = ancestry(parents)
        q_len, base = 5, 3
        query = torch.from_numpy(rng.standard_normal((1, H, q_len, D), dtype=np.float32))
        am = torch.full((1, 1, q_len, PL + cap), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16)
        am[..., :PL + base] = 0
        am[0, 0, :, PL + base:PL + base + q_len] = torch.where(torch.from_numpy(anc), 0.0, torch.finfo(torch.bfloat16).min).to(torch.bfloat16)
        o1, _ = dispatch.unified_forward(None, query, key, val, am, scaling=D ** -0.5)
        arrays["disp_mask_query"] = query.numpy()
        arrays["disp_mask_out"] = o1.numpy()
        arrays["disp_mask_am_bits"] = am.view(torch.int16).numpy().view(np.uint16)
        # causal: one AR token at window position PL + 6 (6 committed before it), window of PL + 7
        q1 = torch.from_numpy(rng.standard_normal((1, H, 1, D), dtype=np.float32))
        o2, _ = dispatch.unified_forward(None, q1, key[:, :, :PL + 7], val[:, :, :PL + 7], None, scaling=D ** -0.5)
        arrays["disp_causal_query"] = q1.numpy()
        arrays["disp_causal_out"] = o2.numpy()
        arrays["disp_kv"] = np.stack([key.numpy(), val.numpy()])
        arrays["disp_stats_kernel"] = np.array(dispatch.STATS["kernel"])
    finally:
        dispatch.uninstall()

    # linear / rmsnorm (fp32 interpreter) and their row invariance.
    x = rng.standard_normal((7, 256), dtype=np.float32)
    w = (rng.standard_normal((192, 256), dtype=np.float32) * 0.05).astype(np.float32)
    y = linear(torch.from_numpy(x), torch.from_numpy(w), BM=32, BN=128, BK=128, num_warps=4, num_stages=3)
    arrays["lin_x"], arrays["lin_w"], arrays["lin_y"] = x, w, y.numpy()
    xn = rng.standard_normal((5, 384), dtype=np.float32)
    wn = rng.uniform(0.5, 1.5, size=384).astype(np.float32)
    arrays["rms_x"], arrays["rms_w"] = xn, wn
    arrays["rms_y"] = rmsnorm(torch.from_numpy(xn), torch.from_numpy(wn), 1e-6).numpy()

    # Eager bf16 RoPE and SiLU*mul (the outputs fused.py's kernels reproduce bitwise).
    from transformers.models.qwen3_vl.modeling_qwen3_vl import rotate_half
    qb = torch.from_numpy(rng.standard_normal((1, 4, 16, 128), dtype=np.float32)).to(torch.bfloat16)
    pos = torch.arange(3000, 3016, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.int64).float() / 128))
    f = pos[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16)[None], emb.sin().to(torch.bfloat16)[None]
    r = qb * cos[:, None] + rotate_half(qb) * sin[:, None]
    arrays["rope_q_bits"] = qb.view(torch.int16).numpy().view(np.uint16)
    arrays["rope_cos_bits"] = cos.view(torch.int16).numpy().view(np.uint16)
    arrays["rope_sin_bits"] = sin.view(torch.int16).numpy().view(np.uint16)
    arrays["rope_out_bits"] = r.view(torch.int16).numpy().view(np.uint16)
    g = torch.from_numpy(rng.standard_normal((4, 512), dtype=np.float32) * 3).to(torch.bfloat16)
    u = torch.from_numpy(rng.standard_normal((4, 512), dtype=np.float32)).to(torch.bfloat16)
    s = torch.nn.functional.silu(g) * u
    arrays["silu_g_bits"] = g.view(torch.int16).numpy().view(np.uint16)
    arrays["silu_u_bits"] = u.view(torch.int16).numpy().view(np.uint16)
    arrays["silu_out_bits"] = s.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(out / "kernels.npz", **arrays)


def candidate_inputs(seed=17):
    """Seeded sentences over a small vocabulary (so keys repeat), lookup prefixes and history frames."""
    rng = np.random.default_rng(seed)
    sent = lambda lo, hi: tuple(int(t) for t in rng.integers(0, 8, int(rng.integers(lo, hi))))
    static = [sent(1, 12) for _ in range(40)]
    drive = [sent(2, 10) for _ in range(12)]
    added = [sent(2, 9) for _ in range(6)]
    prefixes = [[int(t) for t in rng.integers(0, 9, int(rng.integers(0, 5)))] for _ in range(60)]
    frames = [sent(0, 6) for _ in range(14)]
    return dict(static=static, drive=drive, added=added, prefixes=prefixes, frames=frames)


def gen_candidates(out):
    from respect.candidates.datastore import Datastore
    from respect.candidates.history import CocHistory, first_token_filter
    inp = candidate_inputs()
    eos = 8
    res = {"inputs": {k: [list(x) for x in v] for k, v in inp.items()}, "eos": eos, "lookups": [], "history": []}
    def record(gmax, name, d):
        for cmax in (1, 3, 64):
            res["lookups"].append(dict(gmax=gmax, stage=name, cmax=cmax,
                                       out=[[list(c) for c in d.lookup(pfx, cmax)] for pfx in inp["prefixes"]]))

    for gmax in (1, 2, 3):
        ds = Datastore(inp["static"], gmax=gmax).with_drive(inp["drive"])
        record(gmax, "static+drive", ds)            # before the drive index grows
        for s in inp["added"]:
            ds.add(s)
        record(gmax, "after_add", ds)
        record(gmax, "drive_only", ds.without_static())
        record(gmax, "static_only", Datastore(inp["static"], gmax=gmax))
        res.setdefault("num_entries", []).append(Datastore(inp["static"], gmax=gmax).num_entries())
    h = CocHistory(eos)
    for f, s in enumerate(inp["frames"]):
        h.append(f, list(s) + [eos] * (f % 3))
        res["history"].append([[list(c) for c in h.candidates(n)] for n in range(0, 7)])
    cands = [tuple(s) for s in inp["static"][:20]]
    res["first_token"] = [[list(c) for c in first_token_filter(cands, t)] for t in range(10)]
    (out / "candidates.json").write_text(json.dumps(res))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("RESPECT_REF"), required=os.environ.get("RESPECT_REF") is None)
    ap.add_argument("--only", default="trie,verify,kernels,model,candidates")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.ref).resolve()))
    only = set(args.only.split(","))
    torch.manual_seed(0)
    if "trie" in only:
        gen_trie(HERE)
    if "verify" in only:
        gen_verify_mask(HERE)
    if "kernels" in only:
        gen_kernels(HERE)
    if "candidates" in only:
        gen_candidates(HERE)
    if "model" in only:
        sys.path.insert(0, str(HERE))
        import make_model_golden
        make_model_golden.generate(HERE)
    if "token" in only:
        sys.path.insert(0, str(HERE))
        import make_token_golden
        make_token_golden.generate(HERE)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
