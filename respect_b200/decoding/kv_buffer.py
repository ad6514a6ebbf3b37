"""Fixed-capacity KV store for verification rounds, laid out like the native engine.

Drop-in for ``respect.decoding.kv_buffer`` (respect/decoding/kv_buffer.py:20-104):
the public names (``FixedKVBuffer``, ``WindowLayer``, ``WindowCache``,
``compact``) and their contracts are the reference's; the storage is this
package's. One tensor holds the whole model's cache,

    store[layer, 0 | 1, kv_head, slot, dim]      (0 = K, 1 = V)

so ``store[l, 0]`` is exactly the [Hkv, slots, 128] buffer the native engine
reads and writes (``VerifyEngine(kv=buffer)`` runs on it in place), and moving
an accepted path is one native launch over every layer. Slots [0, PL) hold the
prompt, committed tokens follow, then the nodes of the step in flight.

HF models see the store through ``WindowCache`` objects, one per capacity: layer
l of the window with capacity c is a view of the first PL + c slots of
``store[l]``. A forward writes its new keys in place at the slots of its cache
positions. transformers 4.57 passed those positions to the cache layer in
``cache_kwargs["cache_position"]``; 5.x does not, so the window cache also
carries the positions of the forward in flight (``set_positions``, which this
package's ``verify_trie`` and ``forward_tokens`` call) and a layer falls back
to them.
"""
from __future__ import annotations

import ctypes
from typing import Any

import torch
from transformers import cache_utils
from transformers.cache_utils import DynamicCache, DynamicLayer

from respect_b200 import _lib


class WindowLayer(cache_utils.StaticLayer):
    """Layer ``index`` of a FixedKVBuffer's store, seen through its first ``width`` slots."""

    def __init__(self, store: torch.Tensor, index: int, width: int, owner: "WindowCache | None" = None) -> None:
        super().__init__(max_cache_len=width)
        kv = store[index, :, :, :width]                  # [2, Hkv, width, D] view
        self.keys, self.values = kv[0][None], kv[1][None]
        self.owner = owner
        self.max_batch_size, self.num_heads = 1, store.shape[2]
        self.head_dim = store.shape[-1]
        self.dtype, self.device = store.dtype, store.device
        self.is_initialized = True

    def update(self, key_states, value_states, cache_kwargs=None, *args, **kwargs):
        """Write the forward's new K / V at its cache positions; return the whole window."""
        positions = (cache_kwargs or {}).get("cache_position")
        if positions is None and self.owner is not None:
            positions = self.owner.positions
        if positions is None:
            raise RuntimeError("WindowLayer.update: the forward's cache positions are unknown "
                               "(pass cache_position, or call WindowCache.set_positions first)")
        n = key_states.shape[2]
        if positions.numel() != n:
            raise RuntimeError(f"WindowLayer.update: {positions.numel()} cache positions for {n} new keys")
        for dst, src in ((self.keys, key_states), (self.values, value_states)):
            dst.index_copy_(2, positions, src)
        return self.keys, self.values


class WindowCache(cache_utils.Cache):
    """HF cache over one capacity window of a FixedKVBuffer (every layer)."""

    def __init__(self, store: torch.Tensor, width: int) -> None:
        super().__init__(layers=[WindowLayer(store, i, width, self) for i in range(store.shape[0])])
        self.width = width
        self.positions: torch.Tensor | None = None

    def set_positions(self, positions: torch.Tensor | None) -> None:
        """Cache positions (slots) the next forward writes, for transformers that do not pass them."""
        self.positions = positions


class FixedKVBuffer:
    """KV store of a frame: the prompt plus room for ``max(capacities)`` more slots."""

    def __init__(self, prompt_len: int, capacities: tuple[int, ...]) -> None:
        if not capacities:
            raise ValueError("FixedKVBuffer needs at least one capacity")
        self.PL = int(prompt_len)
        self.caps = sorted(int(c) for c in capacities)
        self.store: torch.Tensor | None = None        # [layers, 2, Hkv, slots, D] once allocated
        self._windows: dict[int, WindowCache] = {}

    # ---------------------------------------------------------------- storage
    @property
    def slots(self) -> int:
        return self.PL + self.caps[-1]

    def allocate(self, template: Any) -> None:
        """Allocate the store once, with the layer count, heads, head size, dtype and
        device of a Prefill cache (``template.layers[i].keys`` [1, Hkv, *, D]); later
        calls keep the existing store."""
        if self.store is not None:
            return
        k0 = template.layers[0].keys
        if k0.shape[0] != 1:
            raise ValueError("FixedKVBuffer holds one sequence (batch 1)")
        self.store = torch.zeros((len(template.layers), 2, k0.shape[1], self.slots, k0.shape[3]),
                                 dtype=k0.dtype, device=k0.device)

    def layer_kv(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(K, V) of one layer as [Hkv, slots, D] views: the native engine's buffer layout."""
        return self.store[index, 0], self.store[index, 1]

    @property
    def base_k(self) -> list[torch.Tensor]:
        """Every layer's K as a [1, Hkv, slots, D] view (the reference's per-layer tensors)."""
        return [self.store[i, 0][None] for i in range(self.store.shape[0])]

    @property
    def base_v(self) -> list[torch.Tensor]:
        return [self.store[i, 1][None] for i in range(self.store.shape[0])]

    def write_prefill(self, prefill_cache: Any) -> None:
        """Copy a Prefill cache's first PL slots of every layer into the head of the store."""
        layers = prefill_cache.layers
        if len(layers) != self.store.shape[0]:
            raise ValueError(f"Prefill cache has {len(layers)} layers, the buffer {self.store.shape[0]}")
        for i, layer in enumerate(layers):
            self.store[i, 0, :, :self.PL] = layer.keys[0, :, :self.PL]
            self.store[i, 1, :, :self.PL] = layer.values[0, :, :self.PL]

    # ---------------------------------------------------------------- windows
    def window(self, capacity: int) -> WindowCache:
        """The HF cache that exposes the prompt plus ``capacity`` slots (one object per capacity)."""
        if capacity not in self.caps:
            raise KeyError(f"capacity {capacity} is not one of {self.caps}")
        if capacity not in self._windows:
            self._windows[capacity] = WindowCache(self.store, self.PL + capacity)
        return self._windows[capacity]

    def fit(self, n: int) -> int:
        """The smallest capacity with room for ``n`` slots after the prompt."""
        for c in self.caps:
            if c >= n:
                return c
        raise ValueError(f"no capacity holds {n} slots (capacities {self.caps})")

    def view(self, length: int) -> DynamicCache:
        """A growable HF cache whose layers start as views of the first ``length`` slots
        (nothing is copied; tokens appended later go to new memory, not to the store)."""
        cache = DynamicCache()
        cache.layers = []
        for i in range(self.store.shape[0]):
            layer = DynamicLayer()
            layer.keys = self.store[i, 0, :, :length][None]
            layer.values = self.store[i, 1, :, :length][None]
            layer.dtype, layer.device, layer.is_initialized = self.store.dtype, self.store.device, True
            cache.layers.append(layer)
        return cache

    def compact(self, base: int, path: list[int]) -> None:
        """Move the accepted path's KV to slots PL + base + i, every layer in one launch."""
        compact(self.window(self.caps[-1]), self.PL, base, path)


def compact(cache: Any, prompt_len: int, base: int, slots: list[int]) -> None:
    """Move the KV of an accepted trie path to consecutive slots from ``prompt_len + base``.

    ``slots`` are the path's node indices (strictly increasing), node i having been
    written at slot prompt_len + base + i. One rb_compact_kv launch moves K and V of
    every layer (all layers' tensors must share shape, strides and dtype)."""
    if not len(slots):
        return
    layers = cache.layers
    k0 = layers[0].keys
    b, n_kv, _, d = k0.shape
    if b != 1:
        raise ValueError("compact: batch 1 caches only")
    strides = k0.stride()
    for layer in layers:
        for t in (layer.keys, layer.values):
            if t.shape != k0.shape or t.stride() != strides or t.dtype != k0.dtype:
                raise ValueError("compact: every layer's K and V must share shape, strides and dtype")
    n = len(layers)
    kp = (ctypes.c_void_p * n)(*[layer.keys.data_ptr() for layer in layers])
    vp = (ctypes.c_void_p * n)(*[layer.values.data_ptr() for layer in layers])
    start = prompt_len + base
    src = (ctypes.c_int32 * len(slots))(*[start + int(s) for s in slots])
    _lib.call("rb_compact_kv", kp, vp, n, n_kv, d, strides[1], strides[2], k0.element_size(), src,
              len(slots), start, _lib.stream_of(k0))
