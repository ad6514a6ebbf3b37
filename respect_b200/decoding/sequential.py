"""Token-by-token greedy decoding: the reference that RESPECT must reproduce.

Mirror of ``respect.decoding.sequential`` (respect/decoding/sequential.py:12-42),
on the device of the cache it is given (the reference fixes "cuda"). With the
dedicated kernels installed, each token's logits and KV are bitwise equal to
the same token verified inside a trie.
"""
from __future__ import annotations

import copy
from typing import Any

import torch

from respect_b200.decoding.acceptance import greedy_token


def clone_cache(cache: Any) -> Any:
    """Deep copy of a KV cache so that a run never mutates the shared Prefill state."""
    return copy.deepcopy(cache)


def _device_of(cache: Any, model: Any) -> torch.device:
    layers = getattr(cache, "layers", None)
    if layers and getattr(layers[0], "keys", None) is not None:
        return layers[0].keys.device
    return next(model.vlm.parameters()).device


def forward_tokens(model: Any, token_ids: torch.Tensor, cache: Any, start_position: int) -> tuple[Any, torch.Tensor]:
    dev = _device_of(cache, model)
    positions = torch.arange(start_position, start_position + token_ids.shape[1], device=dev, dtype=torch.long)
    if hasattr(cache, "set_positions"):
        cache.set_positions(positions)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        out = model.vlm(input_ids=token_ids.to(dev), pixel_values=None, past_key_values=cache,
                        cache_position=positions, use_cache=True)
    return out.past_key_values, out.logits.float()


@torch.no_grad()
def sequential(model: Any, cache: Any, token: int, prompt_len: int, eos: int,
               offset: int, size: int, max_tokens: int) -> tuple[list[int], Any]:
    """Generate from ``token`` until EOS or ``max_tokens``, one target run per token.

    ``token`` is the next token to feed (already chosen) and ``cache`` holds the
    KV of everything before it. Returns the generated tokens including ``token``.
    """
    dev = _device_of(cache, model)
    out, pos = [], prompt_len
    while len(out) < max_tokens:
        out.append(token)
        cache, logits = forward_tokens(model, torch.tensor([[token]], device=dev, dtype=torch.long), cache, pos)
        pos += 1
        if token == eos:
            break
        token = int(greedy_token(logits[:, -1, :], offset, size).item())
    return out, cache
