"""Paged GQA decode over 16-token pages.

Drop-in for ``paged_flash_decode(q, k_pool, v_pool, block_table, seq_lens,
page_size)`` (fskernels/paged_attn/triton_paged_attn.py:96-125):
k_pool / v_pool [num_pages, KV_H, 16, 128] (one layer of PagedKVCache's
pools), block_table [B, max_blocks] int32 (-1 = unused), seq_lens [B] int32.
Keyword extras (backward compatible): ``s_aux`` sinks, e4m3 pools with
``scale_k``/``scale_v`` (and an e4m3 q with ``scale_q``), ``out_dtype``, ``out``.
For the same logical KV and lengths the result is bit-identical to the
contiguous entry points.
"""
from __future__ import annotations

import torch

from .. import _native as N
from .. import _ops
from ..gqa_decode import HEAD_DIMS, _check_idx, _check_sink, _inner_contig
from ..gqa_decode_hf import _scale_ptr


def paged_flash_decode(q, k_pool, v_pool, block_table, seq_lens, page_size, *, s_aux=None, scale_q=None,
                       scale_k=None, scale_v=None, out_dtype=None, out=None):
    if q.dim() != 3 or k_pool.dim() != 4 or v_pool.dim() != 4:
        raise ValueError("q must be [B, Q_H, D] and pools [num_pages, KV_H, page_size, D]")
    if not q.is_cuda:
        raise ValueError("paged_flash_decode runs on CUDA tensors only")
    dev = q.device
    if k_pool.device != dev or v_pool.device != dev:
        raise ValueError("q and the pools must be on the same device")
    if k_pool.shape != v_pool.shape or k_pool.dtype != v_pool.dtype:
        raise ValueError("k_pool and v_pool must match in shape and dtype")
    B, QH, D = q.shape
    P, KVH, PS, D2 = k_pool.shape
    if int(page_size) != PS or PS != 16:
        raise ValueError(f"page_size must be 16 and match the pool (pool has {PS})")
    if D not in HEAD_DIMS or D2 != D or (D != 128 and k_pool.element_size() == 1):
        raise ValueError(f"head_dim must be one of {HEAD_DIMS} (128 for an e4m3 pool) and match the pools")
    kv_code = N.dtype_code(k_pool.dtype)
    q_code = N.dtype_code(q.dtype)
    if kv_code != N.FK_DTYPE_E4M3 and q.dtype != k_pool.dtype:
        raise TypeError("q must have the pools' dtype for 16-bit pools")
    if out_dtype is None:
        out_dtype = q.dtype if q.dtype != torch.float8_e4m3fn else torch.float16
    out_code = N.dtype_code(out_dtype)
    q = _inner_contig(q, "q")
    k_pool = _inner_contig(k_pool, "k_pool")
    v_pool = _inner_contig(v_pool, "v_pool")
    if block_table.dim() != 2 or block_table.shape[0] < B:
        raise ValueError("block_table must be [B, max_blocks]")
    bt = block_table
    if bt.device != dev:
        raise ValueError("block_table must be on q's device")
    if bt.dtype != torch.int32 or bt.stride(1) != 1:
        bt = bt.to(torch.int32).contiguous()
    lens = _check_idx(seq_lens, "seq_lens", dev)
    if lens.numel() < B:
        raise ValueError("seq_lens must have one entry per sequence")
    s_aux = _check_sink(s_aux, QH, dev)
    sq = _scale_ptr(scale_q, dev) if q.dtype == torch.float8_e4m3fn else None
    sk = _scale_ptr(scale_k, dev) if kv_code == N.FK_DTYPE_E4M3 else None
    sv = _scale_ptr(scale_v, dev) if kv_code == N.FK_DTYPE_E4M3 else None
    if out is None:
        out = torch.empty(B, QH, D, dtype=out_dtype, device=dev)
    elif out.shape != (B, QH, D) or out.dtype != out_dtype or out.stride(-1) != 1:
        raise ValueError("out must be [B, Q_H, D] of out_dtype with unit inner stride")
    _ops.paged(q, k_pool, v_pool, bt, lens, s_aux, sq, sk, sv, out)
    return out
