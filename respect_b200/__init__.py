"""respect_b200: B200-native (sm_100a) trie-verify hot path of RESPECT.

Operators mirror the reference's modules: ``respect_b200.kernels``
(fused_attn_hyb, linear, rmsnorm, dispatch, patch), ``respect_b200.system.fused``
(rope, silu_mul), ``respect_b200.decoding`` (verify_trie, FixedKVBuffer, compact,
greedy_token, walk, the native VerifyEngine) and ``respect_b200.candidates``
(build_trie, trie_ancestry). All compute runs in librespect_b200.so; there is
no fallback path.
"""
__version__ = "0.1.0"


def load():
    """Load the native library (raises if it is missing)."""
    from respect_b200 import _lib
    return _lib.lib()
