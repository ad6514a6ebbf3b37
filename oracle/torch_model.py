"""One verify forward of a Qwen3-style decoder, restated with torch ops — TEST
INFRASTRUCTURE ONLY (a checker and a CPU baseline, never the product path).

The same algorithm as oracle/model.py (respect/decoding/verify.py:12-46 over
HF's Qwen3VLTextDecoderLayer with the dedicated kernels of
respect/kernels/patch.py:70-107), written with torch tensor ops so that it runs
at BASELINE config-3 size on any device, in one of two modes:

* ``mode="fp32"`` — the oracle's math in fp32 over the given bf16 weights:
  every product accumulates in fp32 and activations are rounded to bf16 at the
  points where the bf16 path rounds (oracle/model.py with bf16=True: after each
  linear, RMSNorm, RoPE product and sum, SiLU, residual add). Attention is the
  exact masked softmax in fp32 over [prefix | committed | trie ancestors]
  (respect/kernels/attention.py:36-71 computes the same function; only the
  order of its fp32 sums differs). This is the full-size reference the GPU
  parity test holds the native engine to.
* ``mode="exact"`` — the same forward with no bf16 rounding of activations at
  all (fp32 throughout over the bf16 weights): the value both bf16
  implementations approximate, against which their errors are measured.
* ``mode="eager"`` — the reference's eager path in bf16, as HF runs it when
  no dedicated kernel is installed (respect/decoding/verify.py:42-46 with
  attention through SDPA and the additive bf16 trie mask of verify.py:35-41):
  bf16 linears, HF RMSNorm (fp32 statistics, cast back, times the weight),
  RoPE and SiLU*mul in bf16, torch's scaled_dot_product_attention. This is
  what bench.py times on the host cores as the CPU baseline.

Weights use the engine's layout (respect_b200.decoding.engine.DecoderWeights):
per layer ``wqkv`` [(H + 2 HK) D, h] (q rows, then k, then v), ``wo`` [h, H D],
``wgu`` [2F, h] with gate and up interleaved in 128-row blocks, ``wd`` [h, F],
norm weights; ``embed`` / ``lm_head`` [V, h], ``final_norm`` [h]. KV: per layer
``kc[l]``, ``vc[l]`` of shape [HK, S, D] (written in place at the node slots).
"""
from __future__ import annotations

import torch


def _round(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> nearest bf16 value (round to nearest even), kept in fp32."""
    return x.to(torch.bfloat16).float() if _ROUND[0] else x


_ROUND = [True]     # False while a mode="exact" forward runs


def _ancestry_mask(parents) -> torch.Tensor:
    """[q, q] bool: row i allows j iff j is i or one of its ancestors
    (respect/candidates/trie.py:53-64); parents precede children."""
    par = [int(p) for p in parents]
    q = len(par)
    out = torch.zeros(q, q, dtype=torch.bool)
    for i in range(q):
        j = i
        while j >= 0:
            out[i, j] = True
            j = par[j]
    return out


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float):
    """bf16 cos/sin [q, D] of the text rotary embedding (all mRoPE axes equal,
    respect/decoding/verify.py:31-33): inv = 1/theta^(2i/D), f = pos*inv, [f, f]."""
    dev = positions.device
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device=dev).float() / head_dim))
    f = positions.float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def _rot(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def _split_gate_up(gu: torch.Tensor):
    """x @ wgu^T [q, 2F] (gate and up in alternating 128-column blocks) -> gate, up [q, F]."""
    q, f2 = gu.shape
    v = gu.view(q, f2 // 256, 2, 128)
    return v[:, :, 0].reshape(q, f2 // 2), v[:, :, 1].reshape(q, f2 // 2)


# --------------------------------------------------------------------- fp32 mode
def _norm32(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm with the oracle's rounding points (respect/kernels/rmsnorm.py:16-21)."""
    var = (x.double() ** 2).mean(-1, keepdim=True).float()
    xh = _round(x * (1.0 / torch.sqrt(var + eps)))
    return _round(w.float() * xh)


def _lin32(x: torch.Tensor, w: torch.Tensor, out_bf16: bool = True) -> torch.Tensor:
    y = x @ w.float().T
    return _round(y) if out_bf16 else y


def _rope32(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    a = _round(x * cos.float())
    r = _round(_rot(x) * sin.float())
    return _round(a + r)


def _attend32(q, k, v, allow, scale):
    """q [H, q, D], k/v [HK, n, D], allow [q, n] bool -> [H, q, D] (fp32 softmax)."""
    G = q.shape[0] // k.shape[0]
    kk = k.repeat_interleave(G, 0)
    vv = v.repeat_interleave(G, 0)
    s = (q @ kk.transpose(1, 2)) * scale
    s = s.masked_fill(~allow[None], float("-inf"))
    return torch.softmax(s, dim=-1) @ vv


# --------------------------------------------------------------------- eager mode
def _norm16(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


@torch.no_grad()
def verify_step(W: dict, cfg: dict, ids, parents, depths, prompt_len: int, base: int, kc, vc,
                mode: str = "fp32", layers: int | None = None) -> torch.Tensor:
    """fp32 logits [q, V] of one verify forward; node i is written to slot
    prompt_len + base + i of every layer's K / V (respect/decoding/verify.py:24-33)."""
    if mode not in ("fp32", "exact", "eager"):
        raise ValueError(f"mode must be 'fp32', 'exact' or 'eager', not {mode!r}")
    if mode == "exact":
        _ROUND[0] = False
        try:
            return verify_step(W, cfg, ids, parents, depths, prompt_len, base, kc, vc, "fp32", layers)
        finally:
            _ROUND[0] = True
    dev = W["embed"].device
    H, HK, D = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    eps, theta = cfg["rms_eps"], cfg["rope_theta"]
    ids = torch.as_tensor(ids, dtype=torch.long, device=dev)
    dep = torch.as_tensor(depths, dtype=torch.long, device=dev)
    q = ids.numel()
    start = prompt_len + base
    slots = torch.arange(start, start + q, device=dev)
    cos, sin = rope_tables(start + dep, D, theta)
    n_keys = start + q
    allow = torch.ones(q, n_keys, dtype=torch.bool)
    allow[:, start:] = _ancestry_mask(list(parents))
    allow = allow.to(dev)
    scale = D ** -0.5
    L = W["layers"] if layers is None else W["layers"][:layers]
    fp32 = mode == "fp32"
    if fp32:
        h = W["embed"][ids].float()
    else:
        h = W["embed"][ids]
        add_mask = torch.zeros(q, n_keys, dtype=torch.bfloat16, device=dev)
        add_mask.masked_fill_(~allow, float("-inf"))
    for li, lw in enumerate(L):
        if fp32:
            qkv = _lin32(_norm32(h, lw["in_norm"], eps), lw["wqkv"])
        else:
            qkv = _norm16(h, lw["in_norm"], eps) @ lw["wqkv"].T
        qh = qkv[:, :H * D].reshape(q, H, D)
        kh = qkv[:, H * D:(H + HK) * D].reshape(q, HK, D)
        vh = qkv[:, (H + HK) * D:].reshape(q, HK, D)
        if fp32:
            qh = _rope32(_norm32(qh, lw["q_norm"], eps).transpose(0, 1), cos[None], sin[None])
            kh = _rope32(_norm32(kh, lw["k_norm"], eps).transpose(0, 1), cos[None], sin[None])
        else:
            qh = _norm16(qh, lw["q_norm"], eps).transpose(0, 1)
            kh = _norm16(kh, lw["k_norm"], eps).transpose(0, 1)
            qh = qh * cos[None] + _rot(qh) * sin[None]
            kh = kh * cos[None] + _rot(kh) * sin[None]
        kc[li][:, slots] = kh.to(kc[li].dtype)
        vc[li][:, slots] = vh.transpose(0, 1).to(vc[li].dtype)
        k_all, v_all = kc[li][:, :n_keys], vc[li][:, :n_keys]
        if fp32:
            a = _attend32(qh, k_all.float(), v_all.float(), allow, scale)
            a = _round(a).transpose(0, 1).reshape(q, H * D)
            h = _round(h + _lin32(a, lw["wo"]))
            x = _norm32(h, lw["post_norm"], eps)
            g, u = _split_gate_up(_lin32(x, lw["wgu"]))
            act = _round(_round(g / (1.0 + torch.exp(-g))) * u)
            h = _round(h + _lin32(act, lw["wd"]))
        else:
            a = torch.nn.functional.scaled_dot_product_attention(
                qh[None], k_all[None], v_all[None], attn_mask=add_mask[None, None], scale=scale, enable_gqa=True)
            a = a[0].transpose(0, 1).reshape(q, H * D)
            h = h + a @ lw["wo"].T
            x = _norm16(h, lw["post_norm"], eps)
            g, u = _split_gate_up(x @ lw["wgu"].T)
            act = torch.nn.functional.silu(g) * u
            h = h + act @ lw["wd"].T
    if fp32:
        return _lin32(_norm32(h, W["final_norm"], eps), W["lm_head"], out_bf16=False)
    return (_norm16(h, W["final_norm"], eps) @ W["lm_head"].T).float()


def weights_of(w) -> dict:
    """The dict this module reads, from a respect_b200 DecoderWeights (same tensors, no copy)."""
    return dict(embed=w.embed, lm_head=w.lm_head, final_norm=w.final_norm, layers=w.layers)


def cfg_of(c) -> dict:
    return dict(n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, rms_eps=c.rms_eps,
                rope_theta=c.rope_theta)


def random_weights_cpu(hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab, seed=0, std=0.02) -> dict:
    """bf16 weights of that architecture on the host, ~N(0, std) elementwise, for
    timing only: each matrix's rows are seeded picks from the rows of one seeded
    N(0, std) pool (drawing 7e9 normals one by one takes minutes on one core; a
    row gather runs at memory speed). Norm weights are 1, as HF initialises them."""
    g = torch.Generator().manual_seed(seed)
    pool = (torch.randn(1 << 24, generator=g) * std).to(torch.bfloat16)

    def mat(n, k):
        rows = pool[: pool.numel() - pool.numel() % k].view(-1, k)
        pick = torch.randint(0, rows.shape[0], (n,), generator=g)
        return rows.index_select(0, pick)

    d = head_dim
    layers = []
    for _ in range(n_layers):
        layers.append(dict(wqkv=mat((n_heads + 2 * n_kv_heads) * d, hidden), wo=mat(hidden, n_heads * d),
                           wgu=mat(2 * ffn, hidden), wd=mat(hidden, ffn),
                           in_norm=torch.ones(hidden, dtype=torch.bfloat16),
                           post_norm=torch.ones(hidden, dtype=torch.bfloat16),
                           q_norm=torch.ones(d, dtype=torch.bfloat16), k_norm=torch.ones(d, dtype=torch.bfloat16)))
    return dict(embed=mat(vocab, hidden), lm_head=mat(vocab, hidden),
                final_norm=torch.ones(hidden, dtype=torch.bfloat16), layers=layers)
