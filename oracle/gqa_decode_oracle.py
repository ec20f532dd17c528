"""CPU oracle for GQA decode attention -- TEST INFRASTRUCTURE ONLY.

This module is the checker the parity tests, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` compare the CUDA kernels against.  The
library itself never imports it: the product path runs only the sm_100a
kernels of ``fasterkernels_b200`` and fails loudly if they are missing.

It restates, in numpy, the reference's torch attention oracle
``ref_attention`` (fskernels/tilelang/tilelang_gqa_decode.py:174-207; the
same formula is copied in tests/test_cuda_fd_gqa.py:16-37 and
tests/test_triton_fd_gqa.py:16-37):

    x_t   = q . k_t / sqrt(D)                         (:191)
    masked positions t >= len get x_t = -inf          (:194-195)
    no sink:  w = softmax(x)                          (:197-198)
    sink s:   M = max(max_t x_t, s)                   (:201-202)
              w_t = e^(x_t - M) / (sum e^(x - M) + e^(s - M))   (:203)
    w is set to 0 on masked positions                 (:205)
    out = sum_t w_t v_t                               (:206)

GQA maps query head qh to KV head qh // G (repeat_kv, :13-22).  A
sequence of length 0 therefore yields an all-zero row (every weight is
masked to 0 at :205).  The paged form follows the layout contract of
fskernels/paged_attn/triton_paged_attn.py:96-125 (pool [P, KVH, 16, D],
logical page p of sequence b at block_table[b, p]); the HF dense form follows
fskernels/triton/triton_gqa_decode_hf.py:44-50 (sequence b attends rows
start_k_offsets[b] .. cache_lens[b]-1).  FP8 inputs are checked, as in
tests/test_triton_gqa_decode_fp8.py:49-53, by running this oracle on the
dequantised K/V (fp8 value x scale).

Parity is pinned by tests/test_oracle_golden.py against vectors produced by
the reference's own ``ref_attention`` and by its Triton kernels run under the
Triton interpreter (tests/golden/make_golden.py).
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "attend_one",
    "decode_varlen",
    "decode_dense",
    "decode_paged",
    "paged_to_dense",
]


def attend_one(q_g, k_t, v_t, sink=None, dtype=np.float64):
    """Attention of G query rows over one KV head's valid tokens.

    q_g [G, D], k_t / v_t [L, D], sink [G] or None -> [G, D].
    Follows tilelang_gqa_decode.py:191-206 for one (sequence, KV head).
    """
    q_g = np.asarray(q_g, dtype=dtype)
    k_t = np.asarray(k_t, dtype=dtype)
    v_t = np.asarray(v_t, dtype=dtype)
    G, D = q_g.shape
    L = k_t.shape[0]
    if L == 0:
        return np.zeros((G, D), dtype=dtype)
    x = (q_g @ k_t.T) * dtype(1.0 / math.sqrt(D))  # [G, L]
    m = x.max(axis=1, keepdims=True)
    if sink is not None:
        s = np.asarray(sink, dtype=dtype).reshape(G, 1)
        m = np.maximum(m, s)
        e = np.exp(x - m)
        w = e / (e.sum(axis=1, keepdims=True) + np.exp(s - m))
    else:
        e = np.exp(x - m)
        w = e / e.sum(axis=1, keepdims=True)
    return w @ v_t


def decode_varlen(q, k_varlen, v_varlen, cu_seqlens, s_aux=None, dtype=np.float64):
    """Varlen decode: q [B, QH, D]; k/v [T, KVH, D]; cu_seqlens [B+1]."""
    q = np.asarray(q)
    B, QH, D = q.shape
    KVH = k_varlen.shape[1]
    G = QH // KVH
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    out = np.zeros((B, QH, D), dtype=dtype)
    for b in range(B):
        lo, hi = int(cu[b]), int(cu[b + 1])
        for h in range(KVH):
            sink = None if s_aux is None else np.asarray(s_aux)[h * G:(h + 1) * G]
            out[b, h * G:(h + 1) * G] = attend_one(
                q[b, h * G:(h + 1) * G], k_varlen[lo:hi, h], v_varlen[lo:hi, h], sink, dtype)
    return out


def decode_dense(q, k_cache, v_cache, cache_lens, start_k_offsets=None, s_aux=None, dtype=np.float64):
    """HF dense-cache decode: k/v [B, KVH, S, D]; rows start..len-1 of sequence b."""
    q = np.asarray(q)
    B, QH, D = q.shape
    KVH, S = k_cache.shape[1], k_cache.shape[2]
    G = QH // KVH
    out = np.zeros((B, QH, D), dtype=dtype)
    for b in range(B):
        hi = min(int(cache_lens[b]), S)
        lo = 0 if start_k_offsets is None else max(int(start_k_offsets[b]), 0)
        lo = min(lo, hi)
        for h in range(KVH):
            sink = None if s_aux is None else np.asarray(s_aux)[h * G:(h + 1) * G]
            out[b, h * G:(h + 1) * G] = attend_one(
                q[b, h * G:(h + 1) * G], k_cache[b, h, lo:hi], v_cache[b, h, lo:hi], sink, dtype)
    return out


def paged_to_dense(k_pool, block_table, seq_lens):
    """Gather a paged pool [P, KVH, PS, D] into per-sequence [KVH, len, D] arrays."""
    PS = k_pool.shape[2]
    seqs = []
    for b, L in enumerate(np.asarray(seq_lens, dtype=np.int64)):
        L = int(L)
        n = (L + PS - 1) // PS
        pages = [k_pool[int(block_table[b, p])] for p in range(n)]  # each [KVH, PS, D]
        if pages:
            full = np.concatenate(pages, axis=1)[:, :L]
        else:
            full = np.zeros((k_pool.shape[1], 0, k_pool.shape[3]), dtype=k_pool.dtype)
        seqs.append(full)
    return seqs


def decode_paged(q, k_pool, v_pool, block_table, seq_lens, s_aux=None, dtype=np.float64):
    """Paged decode over pools [P, KVH, PS, D] and block_table [B, max_blocks]."""
    q = np.asarray(q)
    B, QH, D = q.shape
    KVH = k_pool.shape[1]
    G = QH // KVH
    ks = paged_to_dense(k_pool, block_table, seq_lens)
    vs = paged_to_dense(v_pool, block_table, seq_lens)
    out = np.zeros((B, QH, D), dtype=dtype)
    for b in range(B):
        for h in range(KVH):
            sink = None if s_aux is None else np.asarray(s_aux)[h * G:(h + 1) * G]
            out[b, h * G:(h + 1) * G] = attend_one(q[b, h * G:(h + 1) * G], ks[b][h], vs[b][h], sink, dtype)
    return out
