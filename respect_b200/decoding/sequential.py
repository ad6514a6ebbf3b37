"""Token-by-token greedy decoding on an HF target: the output that RESPECT's trie
verification must reproduce bit for bit.

Drop-in for ``respect.decoding.sequential`` (respect/decoding/sequential.py:12-42;
same names, arguments and results). Built here around a ``TokenStepper``: each
fed token is one target forward of a single query row at the next cache
position, so with the dedicated kernels installed (``kernels.patch``) it runs the
same row-invariant GEMMs, norms and trie attention as a node of a verified trie,
and its logits and KV are the bits a verification commits. The stepper runs on
the device of the cache it is given (the reference fixes "cuda") and names the
forward's write positions to caches that take them (``WindowCache.set_positions``;
transformers 5.x no longer passes them to the cache).
"""
from __future__ import annotations

import copy
import itertools
from typing import Any, Callable, Iterator

import torch

from respect_b200.decoding.acceptance import greedy_token


class TokenStepper:
    """Feeds tokens to ``model.vlm`` one forward at a time, from ``position`` on."""

    def __init__(self, model: Any, cache: Any, position: int) -> None:
        self.model, self.cache, self.position = model, cache, int(position)
        layers = getattr(cache, "layers", None)
        if layers and getattr(layers[0], "keys", None) is not None:
            self.device = layers[0].keys.device
        else:
            self.device = next(model.vlm.parameters()).device

    @torch.no_grad()
    def feed(self, token_ids: torch.Tensor) -> torch.Tensor:
        """One forward over ``token_ids`` [1, n] at the next n positions; returns fp32
        logits [1, n, V] and keeps the updated cache."""
        n = token_ids.shape[1]
        positions = torch.arange(self.position, self.position + n, device=self.device, dtype=torch.long)
        if hasattr(self.cache, "set_positions"):
            self.cache.set_positions(positions)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = self.model.vlm(input_ids=token_ids.to(self.device), pixel_values=None,
                                 past_key_values=self.cache, cache_position=positions, use_cache=True)
        self.cache = out.past_key_values
        self.position += n
        return out.logits.float()

    def greedy_run(self, token: int, eos: int, pick: Callable[[torch.Tensor], int]) -> Iterator[int]:
        """Yield ``token`` and each greedy successor. A token is fed (its KV written)
        before it is yielded; the run ends after feeding ``eos``."""
        while True:
            logits = self.feed(torch.tensor([[token]], dtype=torch.long))
            yield token
            if token == eos:
                return
            token = pick(logits)


def clone_cache(cache: Any) -> Any:
    """An independent copy of a KV cache, so that a decode never changes the shared Prefill state."""
    return copy.deepcopy(cache)


def forward_tokens(model: Any, token_ids: torch.Tensor, cache: Any, start_position: int) -> tuple[Any, torch.Tensor]:
    """One forward of ``token_ids`` [1, n] at positions start_position..; returns (cache, fp32 logits)."""
    stepper = TokenStepper(model, cache, start_position)
    logits = stepper.feed(token_ids)
    return stepper.cache, logits


def sequential(model: Any, cache: Any, token: int, prompt_len: int, eos: int,
               offset: int, size: int, max_tokens: int) -> tuple[list[int], Any]:
    """Decode greedily from ``token`` (already chosen; ``cache`` holds everything before
    it, the first token sitting at position ``prompt_len``) until EOS is fed or
    ``max_tokens`` tokens were fed, one forward per token, excluding the vocabulary
    range [offset, offset + size). Returns the fed tokens (``token`` first) and the cache."""
    stepper = TokenStepper(model, cache, prompt_len)

    def pick(logits: torch.Tensor) -> int:
        return int(greedy_token(logits[:, -1, :], offset, size).item())

    tokens = list(itertools.islice(stepper.greedy_run(token, eos, pick), max(0, max_tokens)))
    return tokens, stepper.cache
