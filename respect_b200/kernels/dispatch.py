"""Route the target's SDPA attention to the trie-verification kernel.

Drop-in for ``respect.kernels.dispatch`` (respect/kernels/dispatch.py:61-140):
``install(PL)`` puts ``unified_forward`` into transformers' attention table
under "sdpa", ``uninstall()`` restores the original. The key axis splits at
the Prompt length PL: slots before PL are the prompt segment, slots from PL on
the node segment. A 4-D mask from the caller is used as is (0 / True opens a
slot); without one the node segment is causal.

Same results as the reference, different plumbing:
  * no padding copies. The reference copies q, the node K/V and a bool mask
    into padded scratch (dispatch.py:94-115) so that its Triton tiles see
    fixed shapes; rb_fused_attn_hyb reads strided views of the window cache
    and of the caller's mask directly (a masked slot is an exact no-op, so
    padding changes nothing) and writes the output straight into the
    [1, q, H, D] layout the caller wants.
  * no fallback. A call the kernel does not cover (batch > 1, dropout,
    attention weights requested, a prompt segment that is not fully open,
    fewer node slots than query rows, shapes the library rejects) raises
    DispatchError; the reference silently ran the original SDPA there
    (dispatch.py:31-32, 116-122). STATS keeps the reference's counters:
    "kernel" counts calls served, "fallback" stays 0, "rejected" counts raises.
"""
from __future__ import annotations

import weakref

import torch
import transformers.integrations.sdpa_attention as SA

from respect_b200 import _lib
from respect_b200.kernels.attention import attn_call

ORIG = SA.sdpa_attention_forward
STATE = {"PL": None}
STATS = {"kernel": 0, "fallback": 0, "rejected": 0}
_PROMPT_OK: dict = {}       # id(mask) -> (weakref to the mask, data_ptr, prompt segment all open)
_PROMPT_CACHE_MAX = 8


class DispatchError(RuntimeError):
    """An attention call outside what the trie kernel computes."""


def _reject(why: str):
    STATS["rejected"] += 1
    raise DispatchError(f"respect_b200 dispatch: {why}")


def _allow(m: torch.Tensor) -> torch.Tensor:
    return m if m.dtype == torch.bool else (m == 0)


def _prompt_all_open(m2: torch.Tensor, am: torch.Tensor, PL: int) -> bool:
    """Whether every query row opens every prompt slot (dispatch.py:50-58).

    The answer is kept per mask tensor (the same object reaches every layer of
    one forward), so a forward pays one device read for it.
    """
    key = id(am)
    hit = _PROMPT_OK.get(key)
    if hit is not None and hit[0]() is am and hit[1] == am.data_ptr():
        return hit[2]
    ok = bool(_allow(m2[:, :PL]).all()) if PL > 0 else True
    if len(_PROMPT_OK) >= _PROMPT_CACHE_MAX:
        _PROMPT_OK.clear()
    _PROMPT_OK[key] = (weakref.ref(am), am.data_ptr(), ok)
    return ok


_KIND = {torch.bool: _lib.RB_MASK_BOOL, torch.uint8: _lib.RB_MASK_BOOL,
         torch.bfloat16: _lib.RB_MASK_ADD_BF16, torch.float32: _lib.RB_MASK_ADD_F32}


def unified_forward(module, query, key, value, attention_mask,
                    dropout=0.0, scaling=None, is_causal=None, **kwargs):
    """query [1, H, q, D], key/value [1, HK, PL + n_node, D] -> ([1, q, H, D], None)."""
    PL = STATE["PL"]
    if PL is None:
        _reject("not installed (call install(prompt_len) first)")
    if query.shape[0] != 1:
        _reject(f"batch {query.shape[0]} (the trie kernel takes one sequence)")
    if dropout != 0.0 or kwargs.get("output_attentions", False):
        _reject("dropout / attention weights are not produced by the trie kernel")
    H, q_len, D = query.shape[1], query.shape[2], query.shape[3]
    HK, n_kv = key.shape[1], key.shape[2]
    n_node = n_kv - PL
    if n_node < q_len:
        _reject(f"{n_kv} keys leave {n_node} node slots for {q_len} query rows (prompt length {PL})")

    msk, kind, first = None, _lib.RB_MASK_CAUSAL, n_node - q_len
    if attention_mask is not None and attention_mask.dim() == 4:
        if attention_mask.shape[-1] != n_kv or attention_mask.shape[-2] != q_len:
            _reject(f"mask {tuple(attention_mask.shape)} does not match {q_len} rows x {n_kv} keys")
        m2 = attention_mask[0, 0]
        if not _prompt_all_open(m2, attention_mask, PL):
            _reject("the mask closes part of the prompt segment")
        msk = m2[:, PL:]
        kind = _KIND.get(msk.dtype)
        if kind is None:           # other additive dtypes: the 0-means-open rule as a bool mask
            msk, kind = (msk == 0), _lib.RB_MASK_BOOL
        elif msk.dtype == torch.bool:
            msk = msk.view(torch.uint8)

    scale = scaling if scaling is not None else D ** -0.5
    out = torch.empty((1, q_len, H, D), dtype=query.dtype, device=query.device)
    k0, v0 = key[0], value[0]
    try:
        attn_call(query[0], k0[:, :PL], v0[:, :PL], k0[:, PL:], v0[:, PL:], msk, out[0].transpose(0, 1), scale,
                  mask_kind=kind, causal_first=first)
    except _lib.RespectNativeError as e:
        _reject(str(e))
    STATS["kernel"] += 1
    return out, None


def install(PL: int) -> None:
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    STATE["PL"] = int(PL)
    _PROMPT_OK.clear()
    SA.sdpa_attention_forward = unified_forward
    ALL_ATTENTION_FUNCTIONS["sdpa"] = unified_forward


def uninstall() -> None:
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    STATE["PL"] = None
    _PROMPT_OK.clear()
    SA.sdpa_attention_forward = ORIG
    ALL_ATTENTION_FUNCTIONS["sdpa"] = ORIG
