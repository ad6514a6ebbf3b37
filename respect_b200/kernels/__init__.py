"""Deterministic kernels of the trie-verify step (mirror of ``respect.kernels``)."""
from respect_b200.kernels.attention import fused_attn_hyb
from respect_b200.kernels.gemm import linear
from respect_b200.kernels.rmsnorm import rmsnorm

__all__ = ["fused_attn_hyb", "linear", "rmsnorm"]
