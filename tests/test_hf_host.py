"""Host-side logic of the HF drop-in (dispatch, patch, FixedKVBuffer) on CPU.

Nothing here computes through the native library: these are the checks that
run before a kernel launch (rejections instead of the reference's silent SDPA
fallback), module installation, the buffer's window/positions bookkeeping, and
that the product path refuses CPU tensors loudly.
"""
import pytest
import torch

from respect_b200.candidates.trie import build_trie
from respect_b200.decoding import kv_buffer
from respect_b200.decoding.verify import verify_trie
from respect_b200.kernels import dispatch, patch


@pytest.fixture(scope="module")
def tiny():
    from tests.golden.make_model_golden import tiny_model

    class Target:
        pass

    t = Target()
    t.vlm = tiny_model(0)
    return t


def _qkv(B=1, H=2, HK=1, q=3, n_kv=10, D=128):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(B, H, q, D, generator=g), torch.randn(B, HK, n_kv, D, generator=g),
            torch.randn(B, HK, n_kv, D, generator=g))


def test_dispatch_rejects_instead_of_falling_back():
    dispatch.install(6)
    try:
        before = dict(dispatch.STATS)
        q, k, v = _qkv(B=2)
        with pytest.raises(dispatch.DispatchError, match="batch"):
            dispatch.unified_forward(None, q, k, v, None)
        q, k, v = _qkv(q=5, n_kv=10)          # 4 node slots for 5 rows
        with pytest.raises(dispatch.DispatchError, match="node slots"):
            dispatch.unified_forward(None, q, k, v, None)
        q, k, v = _qkv(q=3, n_kv=10)
        with pytest.raises(dispatch.DispatchError, match="dropout"):
            dispatch.unified_forward(None, q, k, v, None, dropout=0.1)
        m = torch.zeros(1, 1, 3, 10, dtype=torch.bfloat16)
        m[0, 0, 1, 2] = torch.finfo(torch.bfloat16).min       # closes a prompt slot
        with pytest.raises(dispatch.DispatchError, match="prompt"):
            dispatch.unified_forward(None, q, k, v, m)
        with pytest.raises(dispatch.DispatchError, match="does not match"):
            dispatch.unified_forward(None, q, k, v, torch.zeros(1, 1, 3, 9))
        # a call that passes every check reaches the native library, which refuses CPU tensors
        with pytest.raises(ValueError, match="CUDA"):
            dispatch.unified_forward(None, q, k, v, torch.zeros(1, 1, 3, 10, dtype=torch.bfloat16))
        assert dispatch.STATS["fallback"] == before["fallback"] == 0
        assert dispatch.STATS["rejected"] == before["rejected"] + 5
        assert dispatch.STATS["kernel"] == before["kernel"]
    finally:
        dispatch.uninstall()
    with pytest.raises(dispatch.DispatchError, match="not installed"):
        dispatch.unified_forward(None, *_qkv(), None)


def test_dispatch_prompt_check_is_cached_per_mask():
    dispatch.install(4)
    try:
        m = torch.zeros(1, 1, 2, 8, dtype=torch.bfloat16)
        assert dispatch._prompt_all_open(m[0, 0], m, 4)
        m[0, 0, 0, 1] = -1.0                    # same tensor object: the cached answer stands
        assert dispatch._prompt_all_open(m[0, 0], m, 4)
        m2 = m.clone()                          # a new mask is checked again
        assert not dispatch._prompt_all_open(m2[0, 0], m2, 4)
        b = torch.ones(1, 1, 2, 8, dtype=torch.bool)
        assert dispatch._prompt_all_open(b[0, 0], b, 4)
    finally:
        dispatch.uninstall()


def test_install_swaps_and_restores_modules(tiny):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    lm = patch.language_model(tiny)
    orig = [lm.layers[0].self_attn.q_proj, lm.layers[1].mlp.down_proj, lm.layers[0].input_layernorm,
            lm.layers[1].self_attn.k_norm, lm.norm, tiny.vlm.lm_head]
    n = patch.install(tiny, 40)
    try:
        assert n == 2 * (7 + 4) + 2
        assert patch.is_installed()
        assert isinstance(lm.layers[0].self_attn.q_proj, patch.FixedLinear)
        assert isinstance(lm.layers[1].self_attn.k_norm, patch.FixedNorm)
        assert isinstance(lm.norm, patch.FixedNorm)
        assert tiny.vlm.lm_head.out_dtype == "lm" and lm.layers[0].mlp.up_proj.out_dtype is None
        assert ALL_ATTENTION_FUNCTIONS["sdpa"] is dispatch.unified_forward
        assert patch.install(tiny, 40) == n      # installing twice wraps nothing more
    finally:
        patch.uninstall(tiny)
    assert not patch.is_installed()
    assert ALL_ATTENTION_FUNCTIONS["sdpa"] is dispatch.ORIG
    now = [lm.layers[0].self_attn.q_proj, lm.layers[1].mlp.down_proj, lm.layers[0].input_layernorm,
           lm.layers[1].self_attn.k_norm, lm.norm, tiny.vlm.lm_head]
    assert all(a is b for a, b in zip(orig, now))
    with pytest.raises(RuntimeError):
        with patch.dedicated_kernels(tiny, 40):
            raise RuntimeError("body fails")
    assert not patch.is_installed() and ALL_ATTENTION_FUNCTIONS["sdpa"] is dispatch.ORIG


class _Layer:
    def __init__(self, k, v):
        self.keys, self.values = k, v


class _Cache:
    def __init__(self, layers):
        self.layers = layers


def test_fixed_kv_buffer_windows_and_positions():
    PL, HK, D = 5, 2, 128
    tmpl = _Cache([_Layer(torch.randn(1, HK, PL, D), torch.randn(1, HK, PL, D)) for _ in range(3)])
    buf = kv_buffer.FixedKVBuffer(PL, (16, 8))
    buf.allocate(tmpl)
    buf.allocate(tmpl)                                     # later calls are no-ops
    assert len(buf.base_k) == 3 and buf.base_k[0].shape == (1, HK, PL + 16, D)
    buf.write_prefill(tmpl)
    assert torch.equal(buf.base_k[2][:, :, :PL], tmpl.layers[2].keys)
    assert buf.fit(3) == 8 and buf.fit(9) == 16
    with pytest.raises(ValueError):
        buf.fit(17)
    win = buf.window(8)
    assert win.layers[0].keys.shape[2] == PL + 8
    assert win.layers[0].keys.data_ptr() == buf.base_k[0].data_ptr()
    k_new, v_new = torch.randn(1, HK, 2, D), torch.randn(1, HK, 2, D)
    with pytest.raises(RuntimeError, match="positions"):
        win.layers[1].update(k_new, v_new)
    win.set_positions(torch.tensor([PL + 3, PL + 4]))      # transformers 5.x: positions from the caller
    win.layers[1].update(k_new, v_new)
    assert torch.equal(buf.base_k[1][:, :, PL + 3:PL + 5], k_new)
    win.layers[1].update(v_new, k_new, {"cache_position": torch.tensor([PL, PL + 1])})   # 4.57 style
    assert torch.equal(buf.base_v[1][:, :, PL:PL + 2], k_new)
    view = buf.view(PL + 2)
    assert view.layers[0].keys.shape[2] == PL + 2 and view.layers[0].keys.data_ptr() == buf.base_k[0].data_ptr()
    kv_buffer.compact(win, PL, 0, [])                      # nothing accepted: nothing to do
    with pytest.raises(ValueError, match="CUDA"):          # no CPU path for the move itself
        kv_buffer.compact(win, PL, 0, [0, 2])


def test_verify_trie_host_checks(tiny):
    tree = build_trie([(1, 2, 3), (1, 4)])
    prepared = {"input_ids": torch.zeros(1, 1, dtype=torch.long)}
    with pytest.raises(ValueError, match="capacity"):
        verify_trie(tiny, prepared, None, tree, 10, 2, 5)
    with pytest.raises(ValueError, match="empty"):
        verify_trie(tiny, prepared, None, build_trie([]), 10, 0, 8)
    saved = tiny.vlm.model.rope_deltas
    tiny.vlm.model.rope_deltas = None
    try:
        with pytest.raises(RuntimeError, match="Prefill"):
            verify_trie(tiny, prepared, None, tree, 10, 0, 8)
    finally:
        tiny.vlm.model.rope_deltas = saved
    with pytest.raises(ValueError, match="CUDA"):          # the mask is built by the native library
        verify_trie(tiny, prepared, None, tree, 10, 0, 8)
