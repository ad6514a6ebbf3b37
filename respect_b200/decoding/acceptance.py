"""Greedy token choice and the acceptance walk over a verified trie.

Mirror of ``respect.decoding.acceptance`` (respect/decoding/acceptance.py:11-46).
`greedy_token` runs on the device (rb_greedy_token): the action-vocabulary range
is skipped inside the argmax instead of materialising a masked fp32 clone of
the [q, vocab] logits.
"""
from __future__ import annotations

from typing import Callable

import torch

from respect_b200 import _lib
from respect_b200.candidates.trie import Trie


def mask_action_vocab(logits: torch.Tensor, offset: int, size: int) -> torch.Tensor:
    """fp32 copy of the logits with the trajectory-token range set to -inf."""
    masked = logits.float().clone()
    masked[:, offset:offset + size] = float("-inf")
    return masked


def greedy_token(logits: torch.Tensor, offset: int, size: int) -> torch.Tensor:
    """Row-wise argmax with [offset, offset + size) excluded; int64 [rows] on the logits' device."""
    x = logits if logits.stride(-1) == 1 else logits.contiguous()
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    M, V = x2.shape
    out = torch.empty(M, dtype=torch.int64, device=x.device)
    _lib.call("rb_greedy_token", x2.data_ptr(), _lib.dtype_code(x2.dtype), x2.stride(0), M, V,
              int(offset), int(size), out.data_ptr(), _lib.stream_of(x2))
    return out.reshape(x.shape[:-1])


def walk(tree: Trie, first: int, cap: int, eos: int,
         pick: Callable[[list, int], int]) -> tuple[list, list, int]:
    """Follow the trie from the root holding `first` while each node's token
    matches the target's choice after its parent.

    `pick(accepted, node)` is the target's token after `node`. Stops at EOS, at
    a mismatch, at a leaf, or after `cap` tokens. Returns (node path, accepted
    tokens, correction token): the correction is the target's last choice (or
    `first` when nothing was accepted).
    """
    path: list = []
    accepted: list = []
    correction = first
    node = tree.roots.get(first)
    while node is not None and len(accepted) < cap:
        nd = tree.nodes[node]
        path.append(node)
        accepted.append(nd.token)
        if nd.token == eos:
            break
        correction = pick(accepted, node)
        node = nd.children.get(correction)
    return path, accepted, correction
