"""Install the dedicated kernels into the target language model.

Drop-in for ``respect.kernels.patch`` (respect/kernels/patch.py:1-107): the
seven linear layers of every decoder layer and the vocabulary projection run
rb_linear, the four RMS normalizations of every layer and the final one run
rb_rmsnorm, and SDPA runs the trie kernel through ``dispatch``. Each reduces
in an order fixed by the weight shape alone, so a token's results do not
depend on how many rows (tokens, trie nodes) share the call. The modules are
found where the reference looks for them
(``model.vlm.model.language_model.layers[i].{self_attn,mlp}.*``,
``model.vlm.lm_head``); the vocabulary projection keeps fp32 outputs.
"""
from __future__ import annotations

import contextlib
from typing import Any, Iterator

import torch
import torch.nn as nn

from respect_b200.kernels import dispatch
from respect_b200.kernels.gemm import linear
from respect_b200.kernels.rmsnorm import rmsnorm

LM_OUT_DTYPE = torch.float32  # vocabulary scores are kept in fp32 (patch.py:23)


class FixedLinear(nn.Module):
    def __init__(self, base: nn.Module, out_dtype: str | None = None) -> None:
        super().__init__()
        self.base = base
        self.out_dtype = out_dtype

    def forward(self, x):
        od = LM_OUT_DTYPE if self.out_dtype == "lm" else None
        out = linear(x, self.base.weight, out_dtype=od)
        if getattr(self.base, "bias", None) is not None:
            out = out + self.base.bias
        return out


class FixedNorm(nn.Module):
    def __init__(self, base: nn.Module) -> None:
        super().__init__()
        self.base = base

    def forward(self, x):
        return rmsnorm(x, self.base.weight, self.base.variance_epsilon)


# Modules replaced in every decoder layer: {sub-module ('' = the layer itself): attributes}
PROJECTIONS = {"self_attn": ("q_proj", "k_proj", "v_proj", "o_proj"), "mlp": ("gate_proj", "up_proj", "down_proj")}
NORMS = {"self_attn": ("q_norm", "k_norm"), "": ("input_layernorm", "post_attention_layernorm")}
_saved: list = []   # (owner, attribute, original module), in installation order


def language_model(model: Any):
    inner = model.vlm.model
    return inner.language_model if hasattr(inner, "language_model") else inner


def _replacements(model: Any):
    """(owner, attribute, wrapper) for every module the dedicated kernels take over."""
    lm = language_model(model)
    for layer in lm.layers:
        for table, wrapper in ((PROJECTIONS, FixedLinear), (NORMS, FixedNorm)):
            for sub, attrs in table.items():
                owner = getattr(layer, sub, None) if sub else layer
                for a in attrs:
                    yield owner, a, wrapper
    for a in ("norm", "final_layernorm"):
        if hasattr(getattr(lm, a, None), "variance_epsilon"):
            yield lm, a, FixedNorm
    yield model.vlm, "lm_head", lambda m: FixedLinear(m, "lm")


def is_installed() -> bool:
    return bool(_saved)


def install(model: Any, prompt_len: int) -> int:
    """Wrap the target's linears and norms and route SDPA; returns the number of modules wrapped."""
    for owner, attr, wrapper in _replacements(model):
        cur = getattr(owner, attr, None) if owner is not None else None
        if cur is None or isinstance(cur, (FixedLinear, FixedNorm)):
            continue
        _saved.append((owner, attr, cur))
        setattr(owner, attr, wrapper(cur))
    dispatch.install(prompt_len)
    return len(_saved)


def uninstall(model: Any) -> None:
    dispatch.uninstall()
    while _saved:
        owner, attr, original = _saved.pop()
        setattr(owner, attr, original)


@contextlib.contextmanager
def dedicated_kernels(model: Any, prompt_len: int) -> Iterator[None]:
    """Run the enclosed block with the dedicated kernels installed.

    Install after Prefill: Prefill itself runs on the default kernels.
    """
    install(model, prompt_len)
    try:
        yield
    finally:
        uninstall(model)
