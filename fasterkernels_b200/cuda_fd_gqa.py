"""Positional-sink form of the varlen decode, matching the reference's native
CUDA wrapper ``flash_decode_gqa_varlen(q, k_varlen, v_varlen, cu_seqlens_k,
sink)`` (fskernels/cuda/cuda_fd_gqa.py:14-15)."""
from .gqa_decode import flash_decode_gqa_varlen as _varlen


def flash_decode_gqa_varlen(q, k_varlen, v_varlen, cu_seqlens_k, sink=None):
    return _varlen(q, k_varlen, v_varlen, cu_seqlens_k, sink)
