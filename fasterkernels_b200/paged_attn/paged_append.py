"""Device-side append of one decode token's K/V into a paged pool.

``paged_kv_append`` wraps the C-ABI ``fk_paged_kv_append``: one kernel writes
the new token of every sequence at its device-side position (page
``block_table[b, pos // 16]``, slot ``pos % 16``), quantising to e4m3 with the
pool's per-tensor scales when the pool is float8_e4m3fn.  It replaces the
reference's per-token, per-sequence Python loop with a host sync per token
(fskernels/paged_attn/paged_kv_cache.py:109-132) and is CUDA-graph capturable.
"""
from __future__ import annotations

import torch

from .. import _native as N
from .. import _ops


def paged_kv_append(k_new, v_new, k_pool, v_pool, block_table, positions, *, scale_k=None, scale_v=None,
                    increment: bool = False, status=None):
    """k_new / v_new [B, KV_H, 128] (or [B, KV_H, 1, 128]) float16/bfloat16;
    pools [num_pages, KV_H, 16, 128] of the same dtype or float8_e4m3fn
    (then ``scale_k``/``scale_v`` are 0-dim float32 device tensors);
    block_table [B, max_blocks] int32; positions [B] int32 (device, updated
    in place when ``increment``)."""
    if k_new.dim() == 4:
        k_new, v_new = k_new.squeeze(2), v_new.squeeze(2)
    if k_new.dim() != 3 or k_new.shape != v_new.shape or k_new.shape[-1] not in (64, 128):
        raise ValueError("k_new / v_new must be [B, KV_H, D], D = 128 or 64")
    if not k_new.is_cuda:
        raise ValueError("paged_kv_append runs on CUDA tensors only")
    if (k_pool.dim() != 4 or k_pool.shape != v_pool.shape or k_pool.shape[2] != 16
            or k_pool.shape[3] != k_new.shape[-1]):
        raise ValueError("pools must be [num_pages, KV_H, 16, D] with the head dim of k_new")
    B, KVH, D = k_new.shape
    if k_pool.shape[1] != KVH:
        raise ValueError("pool KV heads do not match k_new")
    if positions.dtype != torch.int32 or positions.numel() < B or not positions.is_contiguous():
        raise TypeError("positions must be a contiguous int32 device tensor with one entry per sequence")
    bt = block_table if (block_table.dtype == torch.int32 and block_table.stride(1) == 1) else \
        block_table.to(torch.int32).contiguous()
    if k_new.stride(-1) != 1:
        k_new = k_new.contiguous()
    if v_new.stride(-1) != 1:
        v_new = v_new.contiguous()
    pool_code = N.dtype_code(k_pool.dtype)
    sk = sv = None
    if pool_code == N.FK_DTYPE_E4M3:
        if scale_k is None or scale_v is None:
            raise ValueError("an e4m3 pool needs scale_k and scale_v")
        sk = scale_k.reshape(()).to(torch.float32).contiguous()
        sv = scale_v.reshape(()).to(torch.float32).contiguous()
    _ops.append(k_new, v_new, k_pool, v_pool, bt, positions, bool(increment), sk, sv, status)
