"""Native verify-step engine (rb_engine_* in include/respect_b200.h).

`VerifyEngine` runs one verify forward of a Qwen3-style decoder over a trie
with the dedicated kernels, natively: what respect/decoding/verify.py:12-46
does through HF with respect/kernels/patch.py:70-107 installed. Weights, KV
buffers and the workspace are torch tensors on one device (torch is the
allocator); every step is a single native call that stages the trie arrays,
replays the CUDA graph of the row bucket and leaves fp32 logits and greedy ids
on the device.

`DecoderConfig.baseline_7b()` is BASELINE.json's config 3 model: hidden 3584,
28 layers, 28 q / 4 kv heads of 128, FFN 18944, vocab 152,064, RoPE theta 1e6.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from respect_b200 import _lib
from respect_b200.candidates.trie import Trie


@dataclass(frozen=True)
class DecoderConfig:
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 1e6

    @staticmethod
    def baseline_7b() -> "DecoderConfig":
        return DecoderConfig(3584, 28, 28, 4, 128, 18944, 152064)

    @staticmethod
    def tiny(n_layers: int = 2) -> "DecoderConfig":
        return DecoderConfig(512, n_layers, 4, 2, 128, 1024, 2048)

    def layer_params(self) -> int:
        d = self.head_dim
        return (self.hidden * (self.n_heads + 2 * self.n_kv_heads) * d + self.n_heads * d * self.hidden
                + 3 * self.hidden * self.ffn + 2 * self.hidden + 2 * d)

    def weight_bytes_per_step(self) -> int:
        """Weights one verify step streams (embedding gather excluded), bf16."""
        return 2 * (self.n_layers * self.layer_params() + self.vocab * self.hidden + self.hidden)


class _LayerW(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("wqkv", "wo", "wgu", "wd", "in_norm", "post_norm", "q_norm", "k_norm")]


class _ModelW(ctypes.Structure):
    _fields_ = [("embed", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("lm_head", ctypes.c_void_p),
                ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
                ("layers", ctypes.POINTER(_LayerW)), ("k_cache", ctypes.POINTER(ctypes.c_void_p)),
                ("v_cache", ctypes.POINTER(ctypes.c_void_p))]


class _Cfg(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("rms_eps", ctypes.c_float), ("max_rows", ctypes.c_int),
                ("max_slots", ctypes.c_int), ("max_pos", ctypes.c_int)]


class _Step(ctypes.Structure):
    _fields_ = [("q", ctypes.c_int), ("base", ctypes.c_int), ("prompt_len", ctypes.c_int),
                ("rope_delta", ctypes.c_int), ("act_off", ctypes.c_int), ("act_size", ctypes.c_int),
                ("ids", ctypes.c_void_p), ("parents", ctypes.c_void_p), ("depths", ctypes.c_void_p),
                ("host_inputs", ctypes.c_int), ("use_graph", ctypes.c_int)]


_ENGINE_SIGS = {
    "rb_engine_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(_Cfg)]),
    "rb_engine_create": (ctypes.c_int, [ctypes.POINTER(_Cfg), ctypes.POINTER(_ModelW), ctypes.c_void_p,
                                        ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "rb_engine_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "rb_engine_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(_Step), ctypes.c_void_p]),
    "rb_engine_outputs": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.c_void_p]),
    "rb_engine_fetch_ids": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "rb_engine_compact": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "rb_engine_accept": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "rb_engine_fetch_accept": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
}
_lib.SIGNATURES.update(_ENGINE_SIGS)


def rope_table(max_pos: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos/sin [max_pos, head_dim] as HF's text rotary embedding produces them
    (inv_freq = 1/theta^(2i/D) in fp32, freqs = pos * inv_freq, emb = [f, f], cast)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim))
    inv = inv.to(device)
    pos = torch.arange(max_pos, dtype=torch.float32, device=device)
    f = pos[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()


class DecoderWeights:
    """bf16 weights in the engine's layout (see rb_layer_weights)."""

    def __init__(self, cfg: DecoderConfig, embed, lm_head, final_norm, layers):
        self.cfg = cfg
        self.embed, self.lm_head, self.final_norm, self.layers = embed, lm_head, final_norm, layers

    @classmethod
    def random(cls, cfg: DecoderConfig, device, seed: int = 0, std: float = 0.02) -> "DecoderWeights":
        """Random init like HF: linears and embedding ~ N(0, std), norm weights 1."""
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        d = cfg.head_dim

        def normal(*shape):
            return torch.empty(shape, dtype=torch.bfloat16, device=device).normal_(0.0, std, generator=g)

        def ones(n):
            return torch.ones(n, dtype=torch.bfloat16, device=device)

        layers = []
        for _ in range(cfg.n_layers):
            layers.append(dict(
                wqkv=normal((cfg.n_heads + 2 * cfg.n_kv_heads) * d, cfg.hidden),
                wo=normal(cfg.hidden, cfg.n_heads * d),
                wgu=normal(2 * cfg.ffn, cfg.hidden),
                wd=normal(cfg.hidden, cfg.ffn),
                in_norm=ones(cfg.hidden), post_norm=ones(cfg.hidden), q_norm=ones(d), k_norm=ones(d)))
        return cls(cfg, normal(cfg.vocab, cfg.hidden), normal(cfg.vocab, cfg.hidden), ones(cfg.hidden), layers)

    @staticmethod
    def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
        """[ffn, hidden] x 2 -> [2 ffn, hidden] in 128-row gate|up blocks."""
        from respect_b200.kernels.gemm import interleave_gate_up
        return interleave_gate_up(gate, up)

    @staticmethod
    def unpack_gate_up(wgu: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        f2, h = wgu.shape
        v = wgu.view(f2 // 256, 2, 128, h)
        return v[:, 0].reshape(f2 // 2, h), v[:, 1].reshape(f2 // 2, h)


class VerifyEngine:
    """One model replica on one device, with its fixed KV buffer.

    The KV buffer has `max_slots` slots per layer ([n_kv_heads, max_slots, 128]
    bf16, a FixedKVBuffer store's per-layer view; the reference's buffer is
    [1, Hkv, PL + cap_max, D] per layer, kv_buffer.py:44-64):
    the prompt occupies [0, prompt_len), committed tokens follow, and a
    verify step writes its nodes after them.
    """

    def __init__(self, weights: DecoderWeights, max_rows: int, max_slots: int | None = None,
                 max_pos: int | None = None, kv=None, share_weights: "VerifyEngine | None" = None):
        """`kv`: an allocated FixedKVBuffer (respect_b200.decoding.kv_buffer) whose store
        [layers, 2, Hkv, slots, D] (bf16) the engine uses as its KV buffer, so a Prefill written
        into it (FixedKVBuffer.write_prefill) is verified in place; max_slots then defaults to
        its slot count. Without it the engine allocates [Hkv, max_slots, D] per layer.
        `share_weights`: another engine of the same model whose packed weights this one
        reuses (several frame streams on one GPU hold the weights once)."""
        self.cfg = c = weights.cfg
        self.w = weights
        self.device = weights.embed.device
        lib = _lib.lib()
        for n, (res, args) in _ENGINE_SIGS.items():
            fn = getattr(lib, n)
            fn.restype, fn.argtypes = res, args
        if kv is not None:
            if kv.store is None:
                raise ValueError("the FixedKVBuffer must be allocated (FixedKVBuffer.allocate) first")
            shape = (c.n_layers, 2, c.n_kv_heads, kv.slots, c.head_dim)
            if (tuple(kv.store.shape) != shape or kv.store.dtype != torch.bfloat16 or not kv.store.is_contiguous()
                    or kv.store.device != self.device):
                raise ValueError(f"KV store must be a contiguous bf16 {shape} tensor on {self.device}, "
                                 f"not {kv.store.dtype} {tuple(kv.store.shape)}")
            max_slots = kv.slots if max_slots is None else max_slots
            if max_slots > kv.slots:
                raise ValueError(f"max_slots {max_slots} exceeds the buffer's {kv.slots} slots")
            pairs = [kv.layer_kv(i) for i in range(c.n_layers)]   # views: the engine writes the store in place
            self.kc = [k for k, _ in pairs]
            self.vc = [v for _, v in pairs]
        else:
            if max_slots is None:
                raise ValueError("max_slots is required without a KV buffer")
            self.kc = [torch.zeros(c.n_kv_heads, max_slots, c.head_dim, dtype=torch.bfloat16, device=self.device)
                       for _ in range(c.n_layers)]
            self.vc = [torch.zeros_like(k) for k in self.kc]
        self.max_rows, self.max_slots = max_rows, max_slots
        self.max_pos = max_pos or (max_slots + 1024)
        self.cos, self.sin = rope_table(self.max_pos, c.head_dim, c.rope_theta, self.device)
        self._cfg = _Cfg(c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab,
                         c.rms_eps, max_rows, max_slots, self.max_pos)
        nbytes = lib.rb_engine_workspace_bytes(ctypes.byref(self._cfg))
        if nbytes == 0:
            raise ValueError(f"respect_b200 engine does not support {c}")
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        # projection weights in the packed tile layout (gate|up with 256-row tiles)
        from respect_b200.kernels.gemm import pack_weight
        if share_weights is not None:
            if share_weights.w is not weights:
                raise ValueError("share_weights must be an engine of the same DecoderWeights")
            self.packed, self.lm_packed = share_weights.packed, share_weights.lm_packed
        else:
            self.packed = [dict(wqkv=pack_weight(lw["wqkv"]), wo=pack_weight(lw["wo"]),
                                wgu=pack_weight(lw["wgu"], 256), wd=pack_weight(lw["wd"])) for lw in weights.layers]
            self.lm_packed = pack_weight(weights.lm_head)
        self._layers = (_LayerW * c.n_layers)(*[
            _LayerW(pk["wqkv"].data_ptr(), pk["wo"].data_ptr(), pk["wgu"].data_ptr(), pk["wd"].data_ptr(),
                    *(lw[k].data_ptr() for k in ("in_norm", "post_norm", "q_norm", "k_norm")))
            for pk, lw in zip(self.packed, weights.layers)])
        self._kp = (ctypes.c_void_p * c.n_layers)(*[t.data_ptr() for t in self.kc])
        self._vp = (ctypes.c_void_p * c.n_layers)(*[t.data_ptr() for t in self.vc])
        mw = _ModelW(weights.embed.data_ptr(), weights.final_norm.data_ptr(), self.lm_packed.data_ptr(),
                     self.cos.data_ptr(), self.sin.data_ptr(), self._layers, self._kp, self._vp)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("rb_engine_create", ctypes.byref(self._cfg), ctypes.byref(mw), self.ws.data_ptr(), nbytes,
                      ctypes.byref(h))
        self._h = h
        lg, ids, hid = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _lib.call("rb_engine_outputs", h, ctypes.byref(lg), ctypes.byref(ids), ctypes.byref(hid), None)
        self._logits_ptr, self._ids_ptr, self._hidden_ptr = lg.value, ids.value, hid.value
        self._ids_host = torch.empty(max_rows, dtype=torch.int64, pin_memory=True)
        self._rec_host = torch.empty(4 + 2 * max_rows, dtype=torch.int32, pin_memory=True)
        self._rec_event = torch.cuda.Event()
        self._rec_n = 0
        self._ids_event = torch.cuda.Event()
        self._ids_n = 0
        self.last_q = 0

    def write_prefill(self, cache, prompt_len: int | None = None) -> None:
        """Copy a Prefill cache (HF Cache or any object with .layers[i].keys / .values of shape
        [1, Hkv, >= prompt_len, D]) into slots [0, prompt_len) (kv_buffer.py:66-71)."""
        layers = cache.layers
        if len(layers) != len(self.kc):
            raise ValueError(f"cache has {len(layers)} layers, the engine {len(self.kc)}")
        for k, v, layer in zip(self.kc, self.vc, layers):
            pl = layer.keys.shape[2] if prompt_len is None else prompt_len
            if pl > self.max_slots:
                raise ValueError(f"prompt of {pl} tokens exceeds max_slots {self.max_slots}")
            k[:, :pl].copy_(layer.keys[0, :, :pl])
            v[:, :pl].copy_(layer.values[0, :, :pl])

    # ------------------------------------------------------------------ steps
    def step(self, ids, parents, depths, base: int, prompt_len: int, rope_delta: int = 0,
             act_off: int = 0, act_size: int = 0, graph: bool = True, stream=None) -> None:
        """Enqueue one verify step. ids/parents/depths: host numpy int32 arrays,
        or int32 CUDA tensors on this engine's device."""
        st = stream or torch.cuda.current_stream(self.device)
        if isinstance(ids, torch.Tensor) and ids.is_cuda:
            ptrs = [t.to(torch.int32).contiguous() for t in (ids, parents, depths)]
            host = 0
        else:
            ptrs = [np.ascontiguousarray(np.asarray(a, dtype=np.int32)) for a in (ids, parents, depths)]
            host = 1
        q = int(ptrs[0].shape[0])
        addr = [p.data_ptr() if isinstance(p, torch.Tensor) else p.ctypes.data for p in ptrs]
        d = _Step(q, base, prompt_len, rope_delta, act_off, act_size, addr[0], addr[1], addr[2], host,
                  1 if graph else 0)
        _lib.call("rb_engine_step", self._h, ctypes.byref(d), st.cuda_stream)
        self._keep = ptrs  # device inputs must outlive the async copy
        self.last_q = q

    def logits(self, q: int | None = None) -> torch.Tensor:
        """fp32 [q, vocab] view of the last step's logits (valid until the next step)."""
        q = self.last_q if q is None else q
        return _view(self._logits_ptr, (q, self.cfg.vocab), torch.float32, self.device)

    def next_ids(self, q: int | None = None) -> torch.Tensor:
        q = self.last_q if q is None else q
        return _view(self._ids_ptr, (q,), torch.int64, self.device)

    def hidden(self, q: int | None = None) -> torch.Tensor:
        q = self.last_q if q is None else q
        return _view(self._hidden_ptr, (q, self.cfg.hidden), torch.bfloat16, self.device)

    def fetch_ids(self, q: int | None = None, stream=None) -> np.ndarray:
        """Greedy ids of the last step, copied to the host (synchronises the stream)."""
        q = self.last_q if q is None else q
        st = stream or torch.cuda.current_stream(self.device)
        _lib.call("rb_engine_fetch_ids", self._h, self._ids_host.data_ptr(), q, st.cuda_stream)
        st.synchronize()
        return self._ids_host[:q].numpy()

    def fetch_ids_async(self, q: int | None = None, stream=None) -> None:
        """Enqueue the copy of the last step's greedy ids to the host; ids_result() waits for it."""
        q = self.last_q if q is None else q
        st = stream or torch.cuda.current_stream(self.device)
        _lib.call("rb_engine_fetch_ids", self._h, self._ids_host.data_ptr(), q, st.cuda_stream)
        self._ids_event.record(st)
        self._ids_n = q

    def ids_result(self) -> np.ndarray:
        self._ids_event.synchronize()
        return self._ids_host[:self._ids_n].numpy().copy()

    def compact(self, path, prompt_len: int, base: int, stream=None) -> None:
        """Move the accepted path's KV to consecutive slots (kv_buffer.py:93-104)."""
        if not len(path):
            return
        st = stream or torch.cuda.current_stream(self.device)
        arr = (ctypes.c_int32 * len(path))(*[int(p) for p in path])
        _lib.call("rb_engine_compact", self._h, arr, len(path), prompt_len, base, st.cuda_stream)

    # ------------------------------------------------------------------ helpers
    def accept(self, first: int, cap: int, eos: int, n: int | None = None, stream=None):
        """The acceptance walk and the KV compaction of the last step, on the device
        (rb_engine_accept): returns (path, tokens, correction) like
        respect_b200.decoding.acceptance.walk, with the accepted KV already moved to
        prompt_len + base + i. n bounds the record read back (default: max_rows)."""
        self.accept_async(first, cap, eos, n, stream)
        return self.accept_result()

    def accept_async(self, first: int, cap: int, eos: int, n: int | None = None, stream=None) -> None:
        """Enqueue the walk, the compaction and the record's copy to the host; the host does
        not wait (several frame streams keep the device busy meanwhile). accept_result()
        waits for the record."""
        st = stream or torch.cuda.current_stream(self.device)
        n = self.max_rows if n is None else n
        if not 0 <= n <= self.max_rows:
            raise ValueError(f"n={n} outside [0, {self.max_rows}]")
        _lib.call("rb_engine_accept", self._h, int(first), int(cap), int(eos), st.cuda_stream)
        _lib.call("rb_engine_fetch_accept", self._h, self._rec_host.data_ptr(), n, st.cuda_stream)
        self._rec_event.record(st)
        self._rec_n = n

    def accept_result(self):
        """(path, tokens, correction) of the last accept_async, after its copy has landed."""
        self._rec_event.synchronize()
        n = self._rec_n
        r = self._rec_host[:4 + 2 * n].tolist()
        cnt = r[0]
        return r[4:4 + cnt], r[4 + n:4 + n + cnt], r[1]

    def verify(self, tree: Trie, prompt_len: int, base: int, act_off: int = 0, act_size: int = 0,
               graph: bool = True) -> np.ndarray:
        """verify_trie + greedy_token for a host trie: returns the greedy ids per node (host)."""
        self.step(tree.tokens().astype(np.int32), tree.parents(), tree.depths(), base, prompt_len,
                  act_off=act_off, act_size=act_size, graph=graph)
        return self.fetch_ids(len(tree.nodes))

    def prefill(self, tokens, chunk: int | None = None, graph: bool = True, reuse=None, stream=None) -> int:
        """Fill KV slots [0, len(tokens)) by running the prompt in chunks: chunk c is a
        linear chain whose prompt is the c * chunk tokens before it (prompt_len = c * chunk,
        base 0), so the earlier chunks are read by the prefix phase of the attention.

        `reuse`: the tokens whose KV the buffer holds now (the previous frame's prompt,
        prefilled with the same chunk). The chunks that lie entirely before the first
        token that differs are kept: a slot's KV depends only on the tokens up to it and
        the chunk grid, so the kept slots equal a recompute bitwise. Returns the number
        of tokens recomputed (at least the last chunk, whose last row's greedy pick, in
        next_ids(), is the token after the prompt)."""
        chunk = chunk or self.max_rows
        toks = np.asarray(tokens, np.int32)
        if len(toks) > self.max_slots:
            raise ValueError(f"prompt of {len(toks)} tokens exceeds max_slots {self.max_slots}")
        start = prefill_start(toks, reuse, chunk)
        for s in range(start, len(toks), chunk):
            part = toks[s:s + chunk]
            n = len(part)
            self.step(part, np.arange(-1, n - 1, dtype=np.int32), np.arange(n, dtype=np.int32), 0, s,
                      graph=graph, stream=stream)
        return len(toks) - start

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().rb_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def prefill_start(tokens, reuse, chunk: int) -> int:
    """First prompt position a chunked prefill recomputes when the buffer holds the KV of
    `reuse` (prefilled with the same chunk): the start of the chunk holding the first
    token that differs, but no later than the start of the last chunk (which always runs:
    its last row's greedy pick is the token after the prompt). 0 without `reuse`."""
    toks = np.asarray(tokens)
    if reuse is None or len(toks) == 0:
        return 0
    if chunk <= 0:
        raise ValueError(f"chunk must be positive, got {chunk}")
    old = np.asarray(reuse)
    n = min(len(old), len(toks))
    diff = np.flatnonzero(old[:n] != toks[:n])
    lcp = int(diff[0]) if len(diff) else n
    return min((lcp // chunk) * chunk, ((len(toks) - 1) // chunk) * chunk)


def _view(ptr: int, shape, dtype, device) -> torch.Tensor:
    """Non-owning torch view of engine-workspace memory."""
    n = 1
    for s in shape:
        n *= s
    esize = torch.empty((), dtype=dtype).element_size()

    class _Holder:
        __cuda_array_interface__ = {
            "shape": (n,), "typestr": {torch.float32: "<f4", torch.int64: "<i8", torch.bfloat16: "<u2"}[dtype],
            "data": (ptr, False), "version": 3, "strides": None}

    t = torch.as_tensor(_Holder(), device=device)
    if dtype == torch.bfloat16:
        t = t.view(torch.bfloat16)
    return t.view(*shape)
