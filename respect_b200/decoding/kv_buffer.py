"""Fixed-capacity KV buffer shared by initial and follow-up verification.

Mirror of ``respect.decoding.kv_buffer`` (respect/decoding/kv_buffer.py:1-104):
one buffer per layer, [1, HK, PL + max(capacities), D], allocated once and
reused across frames; a window exposes its first PL + capacity slots to a
forward pass and new keys are written in place at the forward's cache
positions; after a verification ``compact`` moves the accepted path's KV to
consecutive slots so the next forward reads what a sequential run would.

The write positions: transformers 4.57 hands them to the cache layer in
``cache_kwargs["cache_position"]``; transformers 5.x no longer passes them, so
the window cache also carries the positions of the forward in flight
(``WindowCache.set_positions``; ``verify_trie`` and ``forward_tokens`` set
them) and a layer uses them when the call brings none.

``compact`` is one native launch (rb_compact_kv) for all layers' K and V,
where the reference issues an index_select + index_copy_ pair per tensor.
"""
from __future__ import annotations

import ctypes
from typing import Any

import torch
from transformers import cache_utils
from transformers.cache_utils import DynamicCache, DynamicLayer

from respect_b200 import _lib


class WindowLayer(cache_utils.StaticLayer):
    """One layer of the shared buffer, exposing only its first ``window`` slots."""

    def __init__(self, base_k: torch.Tensor, base_v: torch.Tensor, window: int, owner: "WindowCache" = None) -> None:
        super().__init__(max_cache_len=window)
        self._base_k, self._base_v, self._window = base_k, base_v, window
        self._owner = owner
        self.keys = base_k[:, :, :window, :]
        self.values = base_v[:, :, :window, :]
        self.max_batch_size, self.num_heads, _, self.head_dim = base_k.shape
        self.dtype, self.device = base_k.dtype, base_k.device
        self.is_initialized = True

    def update(self, key_states, value_states, cache_kwargs=None, *args, **kwargs):
        pos = (cache_kwargs or {}).get("cache_position")
        if pos is None:
            pos = self._owner.positions if self._owner is not None else None
        if pos is None:
            raise RuntimeError("WindowLayer.update: no cache positions (set them with WindowCache.set_positions)")
        if pos.numel() != key_states.shape[2]:
            raise RuntimeError(f"WindowLayer.update: {pos.numel()} positions for {key_states.shape[2]} new keys")
        self.keys.index_copy_(2, pos, key_states)
        self.values.index_copy_(2, pos, value_states)
        return self.keys, self.values


class WindowCache(cache_utils.Cache):
    def __init__(self, layers: list = None, bases: list = None, window: int = 0) -> None:
        if layers is None:
            layers = [WindowLayer(bk, bv, window, self) for bk, bv in bases]
        super().__init__(layers=layers)
        self.positions = None

    def set_positions(self, positions: torch.Tensor | None) -> None:
        """Slots the next forward writes (its cache_position), for transformers that do not pass them."""
        self.positions = positions


class FixedKVBuffer:
    def __init__(self, prompt_len: int, capacities: tuple[int, ...]) -> None:
        self.PL = prompt_len
        self.caps = sorted(capacities)
        self.base_k: list[torch.Tensor] = []
        self.base_v: list[torch.Tensor] = []
        self.caches: dict[int, WindowCache] = {}

    def allocate(self, template: Any) -> None:
        """Allocate once, shaped after a Prefill cache. Later calls are no-ops."""
        if self.base_k:
            return
        slots = self.PL + self.caps[-1]
        for layer in template.layers:
            b, h, _, d = layer.keys.shape
            self.base_k.append(torch.zeros((b, h, slots, d), dtype=layer.keys.dtype, device=layer.keys.device))
            self.base_v.append(torch.zeros((b, h, slots, d), dtype=layer.keys.dtype, device=layer.keys.device))
        bases = list(zip(self.base_k, self.base_v))
        self.caches = {cap: WindowCache(bases=bases, window=self.PL + cap) for cap in self.caps}

    def write_prefill(self, prefill_cache: Any) -> None:
        """Copy the Prefill KV into the head of the buffer (done once per frame)."""
        PL = self.PL
        for bk, bv, layer in zip(self.base_k, self.base_v, prefill_cache.layers):
            bk[:, :, :PL].copy_(layer.keys[..., :PL, :])
            bv[:, :, :PL].copy_(layer.values[..., :PL, :])

    def window(self, capacity: int) -> WindowCache:
        return self.caches[capacity]

    def fit(self, n: int) -> int:
        """Smallest capacity that holds ``n`` slots."""
        for c in self.caps:
            if c >= n:
                return c
        raise ValueError(f"no capacity holds {n} slots (capacities {self.caps})")

    def view(self, length: int) -> DynamicCache:
        """A cache that sees the first ``length`` slots without copying."""
        c = DynamicCache()
        c.layers = []
        for bk, bv in zip(self.base_k, self.base_v):
            layer = DynamicLayer()
            layer.keys, layer.values = bk[:, :, :length], bv[:, :, :length]
            layer.dtype, layer.device, layer.is_initialized = bk.dtype, bk.device, True
            c.layers.append(layer)
        return c


def compact(cache: Any, prompt_len: int, base: int, slots: list[int]) -> None:
    """Move the KV of the accepted path to consecutive slots starting at ``prompt_len + base``.

    ``slots`` are node indices of an accepted trie path (strictly increasing),
    node i living at slot prompt_len + base + i.
    """
    if not slots:
        return
    layers = cache.layers
    k0 = layers[0].keys
    b, HK, S, D = k0.shape
    if b != 1:
        raise ValueError("compact: batch 1 caches only")
    strides = k0.stride()
    for layer in layers:
        for t in (layer.keys, layer.values):
            if t.shape != k0.shape or t.stride() != strides or t.dtype != k0.dtype:
                raise ValueError("compact: every layer's K and V must share shape, strides and dtype")
    n_layers = len(layers)
    kp = (ctypes.c_void_p * n_layers)(*[layer.keys.data_ptr() for layer in layers])
    vp = (ctypes.c_void_p * n_layers)(*[layer.values.data_ptr() for layer in layers])
    start = prompt_len + base
    src = (ctypes.c_int32 * len(slots))(*[start + int(s) for s in slots])
    _lib.call("rb_compact_kv", kp, vp, n_layers, HK, D, strides[1], strides[2], k0.element_size(), src,
              len(slots), start, _lib.stream_of(k0))
