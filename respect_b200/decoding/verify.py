"""One target run that verifies every node of a trie.

Mirror of ``respect.decoding.verify.verify_trie`` (respect/decoding/verify.py:12-46):
node i is written to slot prompt_len + base + i (its physical slot) while its
rotary position follows its depth in the trie (its logical position); the
additive bf16 mask [1, 1, q, prompt_len + capacity] opens the prompt and the
committed tokens to every node and each node to its ancestors-or-self.

The mask is written on the device by rb_verify_mask from the parent array
(the reference fills it with torch ops from a host-built [q, q] ancestry);
the node ids, depths and parents cross to the device in one copy.
"""
from __future__ import annotations

from typing import Any

import torch

from respect_b200 import _lib


def trie_inputs(tree, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(ids [1, q] int64, depths [q] int64, parents [q] int32) on ``device``, from one host->device copy."""
    nodes = tree.nodes
    q = len(nodes)
    host = torch.empty((3, q), dtype=torch.int64, pin_memory=torch.cuda.is_available())
    host[0] = torch.tensor([n.token for n in nodes], dtype=torch.int64)
    host[1] = torch.tensor([n.depth for n in nodes], dtype=torch.int64)
    host[2] = torch.tensor([-1 if n.parent is None else n.parent for n in nodes], dtype=torch.int64)
    dev = host.to(device, non_blocking=True)
    return dev[0].view(1, q), dev[1], dev[2].to(torch.int32)


def verify_mask(parents: torch.Tensor, prompt_len: int, base: int, capacity: int) -> torch.Tensor:
    """Additive bf16 mask [1, 1, q, prompt_len + capacity] (verify.py:35-41)."""
    q = parents.numel()
    width = prompt_len + capacity
    m = torch.empty((1, 1, q, width), dtype=torch.bfloat16, device=parents.device)
    _lib.call("rb_verify_mask", parents.data_ptr(), q, prompt_len + base, width, m.data_ptr(),
              _lib.stream_of(parents))
    return m


@torch.no_grad()
def verify_trie(model: Any, prepared: dict, cache: Any, tree: Any,
                prompt_len: int, base: int, capacity: int) -> Any:
    """Verify all trie nodes in one forward pass on the fixed-capacity cache."""
    dev = prepared["input_ids"].device
    q = len(tree.nodes)
    start = prompt_len + base
    if q == 0:
        raise ValueError("verify_trie: empty trie")
    if base + q > capacity:
        raise ValueError(f"verify_trie: {q} nodes after {base} committed tokens exceed capacity {capacity}")
    rope = getattr(model.vlm.model, "rope_deltas", None)
    if rope is None:
        raise RuntimeError("rope_deltas is missing; verify only after Prefill")
    ids, depth, parents = trie_inputs(tree, dev)
    cache_position = torch.arange(start, start + q, device=dev)
    delta = start + rope.to(device=dev, dtype=torch.long).reshape(-1)[:1]
    logical = (depth + delta).view(1, 1, q).expand(3, -1, -1)
    mask = verify_mask(parents, prompt_len, base, capacity)
    if hasattr(cache, "set_positions"):
        cache.set_positions(cache_position)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        return model.vlm(input_ids=ids, pixel_values=None, past_key_values=cache,
                         cache_position=cache_position, position_ids=logical,
                         attention_mask=mask, use_cache=True, return_dict=True,
                         output_hidden_states=True)
