"""GQA varlen flash-decode with optional attention sinks (contiguous KV).

Drop-in for ``flash_decode_gqa_varlen`` of the reference
(fskernels/triton/triton_gqa_decode.py:126-155, and the native variant
fskernels/cuda/cuda_fd_gqa.py:14-15 whose fifth argument is positional).
Differences that keep the contract but fix the reference's behaviour:
  * the sink follows the reference's torch oracle
    (fskernels/tilelang/tilelang_gqa_decode.py:198-203), not the raw
    ``l += s_aux`` of its kernels (triton_gqa_decode.py:112-115);
  * no host synchronisation (the reference computes ``int(max(len))`` on the
    host, triton_gqa_decode.py:135), so the call can be captured in a CUDA
    graph;
  * sequences are split across the whole GPU on the device (stream-K over
    16-token granules) instead of one CTA per (sequence, KV head).
"""
from __future__ import annotations

import torch

from . import _native as N  # noqa: F401  (loads the library on first use)
from . import _ops

HEAD_DIM = 128
HEAD_DIMS = (64, 128)  # 64 with float16/bfloat16 KV only


def _inner_contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.stride(-1) != 1:
        t = t.contiguous()
    return t


def _check_sink(s_aux, q_heads: int, device) -> torch.Tensor | None:
    if s_aux is None:
        return None
    if s_aux.device != device:
        raise ValueError("s_aux must be on the same device as q")
    if s_aux.numel() != q_heads:
        raise ValueError(f"s_aux must have q_heads={q_heads} elements, got {s_aux.numel()}")
    if s_aux.dtype != torch.float32 or not s_aux.is_contiguous():
        s_aux = s_aux.reshape(-1).to(torch.float32).contiguous()
    return s_aux


def _check_idx(t: torch.Tensor, name: str, device) -> torch.Tensor:
    if t.device != device:
        raise ValueError(f"{name} must be on the same device as q")
    if t.dtype != torch.int32 or not t.is_contiguous():
        t = t.to(torch.int32).contiguous()
    return t


def flash_decode_gqa_varlen(q, k_varlen, v_varlen, cu_seqlens_k, s_aux=None, *, out=None):
    """out[b, qh] = attention of q[b, qh] over k/v rows cu_seqlens_k[b]..cu_seqlens_k[b+1]-1
    of KV head qh // G, with the optional per-query-head sink logit s_aux[qh].

    q [B, Q_H, D], k_varlen / v_varlen [T, KV_H, D] (float16 or bfloat16,
    D = 128 or 64), cu_seqlens_k [B+1] int32, s_aux [Q_H] float32 or None.
    Returns [B, Q_H, D].
    """
    if q.dim() != 3 or k_varlen.dim() != 3 or v_varlen.dim() != 3:
        raise ValueError("q must be [B, Q_H, D] and k_varlen/v_varlen [T, KV_H, D]")
    if not q.is_cuda:
        raise ValueError("flash_decode_gqa_varlen runs on CUDA tensors only")
    dev = q.device
    if k_varlen.device != dev or v_varlen.device != dev:
        raise ValueError("q, k_varlen and v_varlen must be on the same device")
    if not (q.dtype == k_varlen.dtype == v_varlen.dtype):
        raise TypeError("q, k_varlen and v_varlen must share one dtype")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("flash_decode_gqa_varlen takes float16 or bfloat16 tensors")
    B, QH, D = q.shape
    T, KVH, D2 = k_varlen.shape
    if D not in HEAD_DIMS or D2 != D or v_varlen.shape != k_varlen.shape:
        raise ValueError(f"head_dim must be one of {HEAD_DIMS} and q/k/v head dims and k/v shapes must match")
    if cu_seqlens_k.numel() != B + 1:
        raise ValueError("cu_seqlens_k must have batch + 1 entries")
    q = _inner_contig(q, "q")
    k_varlen = _inner_contig(k_varlen, "k_varlen")
    v_varlen = _inner_contig(v_varlen, "v_varlen")
    cu = _check_idx(cu_seqlens_k, "cu_seqlens_k", dev)
    s_aux = _check_sink(s_aux, QH, dev)
    if out is None:
        out = torch.empty(B, QH, D, dtype=q.dtype, device=dev)
    elif out.shape != (B, QH, D) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must be [B, Q_H, D] of q's dtype with unit inner stride")
    _ops.varlen(q, k_varlen, v_varlen, cu, s_aux, out)
    return out
