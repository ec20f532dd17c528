"""HF dense-cache GQA decode and the Hugging Face attention adapter.

Drop-in for fskernels/triton/triton_gqa_decode_hf.py:
  * ``set_num_splits`` (:12-14) -- kept for CUDAGraphRunner
    (fskernels/engine/cuda_graph_runner.py:175-176).  The split count here is
    planned on the device from the sequence lengths, so the value is recorded
    (``get_num_splits``) and accepted but does not change the result or the
    schedule.
  * ``flash_decode_gqa_hf_dense_optimized(q, k_cache, v_cache, cache_lens,
    start_k_offsets=None, num_splits=None)`` (:146-211): sequence b attends
    cache rows start_k_offsets[b] .. cache_lens[b]-1 (:44-50).  Partials are
    kept in fp32 (the reference stores them in the output dtype, :182).
  * ``custom_hf_decode_attention_forward`` (:218-258): q_len == 1 with a cache
    and ``cache_position`` -> the sm_100a kernel; anything else -> the
    transformers eager attention, exactly as the reference routes prefill.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _native as N
from . import _ops
from .gqa_decode import HEAD_DIMS, _check_idx, _check_sink, _inner_contig

_DECODE_NUM_SPLITS: int = 1


def set_num_splits(n: int) -> None:
    global _DECODE_NUM_SPLITS
    n = int(n)
    if n < 1:
        raise ValueError("num_splits must be >= 1")
    _DECODE_NUM_SPLITS = n


def get_num_splits() -> int:
    return _DECODE_NUM_SPLITS


def _scale_ptr(x, dev):
    if x is None:
        return None
    if not torch.is_tensor(x):
        x = torch.tensor(float(x), dtype=torch.float32, device=dev)
    if x.device != dev:
        raise ValueError("FP8 scales must be device tensors on q's device")
    if x.dtype != torch.float32 or not x.is_contiguous():
        x = x.reshape(()).to(torch.float32).contiguous()
    return x


def dense_decode(q, k_cache, v_cache, cache_lens, start_k_offsets=None, *, s_aux=None, scale_q=None,
                 scale_k=None, scale_v=None, out_dtype=None, out=None):
    """Core HF-dense entry: k/v [B, KV_H, S, 128] in float16/bfloat16 (q the same
    dtype) or float8_e4m3fn (q float16/bfloat16, or float8_e4m3fn with scale_q)."""
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("q must be [B, Q_H, D] and k/v caches [B, KV_H, S, D]")
    if not q.is_cuda:
        raise ValueError("dense decode runs on CUDA tensors only")
    dev = q.device
    if k_cache.device != dev or v_cache.device != dev:
        raise ValueError("q and the caches must be on the same device")
    if k_cache.dtype != v_cache.dtype or k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must match in shape and dtype")
    B, QH, D = q.shape
    Bk, KVH, S, D2 = k_cache.shape
    if D not in HEAD_DIMS or D2 != D or (D != 128 and k_cache.element_size() == 1):
        raise ValueError(f"head_dim must be one of {HEAD_DIMS} (128 for an e4m3 cache) and match the cache")
    if Bk < B:
        raise ValueError("cache batch is smaller than q's batch")
    kv_code = N.dtype_code(k_cache.dtype)
    q_code = N.dtype_code(q.dtype)
    if out_dtype is None:
        out_dtype = q.dtype if q.dtype != torch.float8_e4m3fn else torch.float16
    out_code = N.dtype_code(out_dtype)
    q = _inner_contig(q, "q")
    k_cache = _inner_contig(k_cache, "k_cache")
    v_cache = _inner_contig(v_cache, "v_cache")
    lens = _check_idx(cache_lens, "cache_lens", dev)
    if lens.numel() < B:
        raise ValueError("cache_lens must have one entry per sequence")
    starts = None if start_k_offsets is None else _check_idx(start_k_offsets, "start_k_offsets", dev)
    s_aux = _check_sink(s_aux, QH, dev)
    sq = _scale_ptr(scale_q, dev) if q.dtype == torch.float8_e4m3fn else None
    sk = _scale_ptr(scale_k, dev) if kv_code == N.FK_DTYPE_E4M3 else None
    sv = _scale_ptr(scale_v, dev) if kv_code == N.FK_DTYPE_E4M3 else None
    if out is None:
        out = torch.empty(B, QH, D, dtype=out_dtype, device=dev)
    elif out.shape != (B, QH, D) or out.dtype != out_dtype or out.stride(-1) != 1:
        raise ValueError("out must be [B, Q_H, D] of out_dtype with unit inner stride")
    _ops.dense(q, k_cache, v_cache, lens, starts, s_aux, sq, sk, sv, out)
    return out


def flash_decode_gqa_hf_dense_optimized(q, k_cache, v_cache, cache_lens, start_k_offsets=None, num_splits=None,
                                        *, s_aux=None, out=None):
    """Decode over an HF BHSD cache.  ``num_splits`` is accepted for API
    compatibility; the split schedule is planned on the device."""
    if num_splits is not None and int(num_splits) < 1:
        raise ValueError("num_splits must be >= 1")
    if q.dtype not in (torch.float16, torch.bfloat16) or k_cache.dtype != q.dtype:
        raise TypeError("flash_decode_gqa_hf_dense_optimized takes float16/bfloat16 q and caches of q's dtype")
    return dense_decode(q, k_cache, v_cache, cache_lens, start_k_offsets, s_aux=s_aux, out=out)


def _module_sinks(module, q_heads, dev):
    sinks = getattr(module, "sinks", None)
    if sinks is None or not torch.is_tensor(sinks) or sinks.numel() != q_heads:
        return None
    return sinks.detach().to(device=dev, dtype=torch.float32).reshape(-1)


def _decode_window(kwargs, bsz, dev, attention_mask=None, cache_len=None):
    """(cache_lens, start offsets or None) for a q_len == 1 call, with tensor
    ops only (graph-safe).
    * ``cache_position`` given (the reference's runner passes it,
      fskernels/engine/cuda_graph_runner.py:193,211): length = position + 1,
      as triton_gqa_decode_hf.py:239-242 computes it; a ``sliding_window``
      gives the window [max(0, len - window), len).
    * otherwise (transformers 5.x no longer passes ``cache_position``): the
      attended range of each row is the span of its valid mask positions
      (left padding becomes a start offset), or the whole cache without a mask.
    """
    cache_position = kwargs.get("cache_position")
    starts = None
    if cache_position is not None:
        lens = (cache_position[-1:] + 1).to(torch.int32).expand(bsz).contiguous()
    elif attention_mask is not None:
        m = attention_mask.reshape(attention_mask.shape[0], -1)[:, -int(cache_len):]
        valid = m if m.dtype == torch.bool else (m == 0)
        valid = valid.expand(bsz, -1)
        S = valid.shape[1]
        first = torch.argmax(valid.to(torch.int32), dim=1)
        last = S - torch.argmax(valid.flip(1).to(torch.int32), dim=1)
        any_valid = valid.any(dim=1)
        lens = torch.where(any_valid, last, torch.zeros_like(last)).to(torch.int32).contiguous()
        starts = torch.where(any_valid, first, torch.zeros_like(first)).to(torch.int32).contiguous()
    else:
        lens = torch.full((bsz,), int(cache_len), dtype=torch.int32, device=dev)
    window = kwargs.get("sliding_window")
    if window is not None:
        wstart = torch.clamp(lens - int(window), min=0).to(torch.int32)
        starts = wstart if starts is None else torch.maximum(starts, wstart)
    return lens, starts


def _fallback(module, query_states, key_states, value_states, attention_mask, scaling, dropout, **kwargs):
    """Prefill / non-decode calls: transformers' own SDPA attention (the
    reference falls back to the native eager attention the same way,
    triton_gqa_decode_hf.py:256-258)."""
    try:
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        return sdpa_attention_forward(module, query_states, key_states, value_states, attention_mask,
                                      scaling=scaling, dropout=dropout, **kwargs)
    except ImportError:  # pragma: no cover
        from transformers.models.qwen3.modeling_qwen3 import eager_attention_forward
        return eager_attention_forward(module, query_states, key_states, value_states, attention_mask, scaling,
                                       dropout, **kwargs)


def _check_scaling(scaling, head_dim):
    """The kernels scale logits by head_dim ** -0.5, as the reference's HF
    adapters do whatever ``scaling`` says (triton_gqa_decode_hf.py:50).  A
    model whose attention uses another scale would get wrong attention, so
    such a call is refused instead of silently decoded."""
    if scaling is None:
        return
    want = float(head_dim) ** -0.5
    if abs(float(scaling) - want) > 1e-4 * want:
        raise ValueError(f"attention scaling {float(scaling)!r} is not head_dim**-0.5 = {want!r}; the decode "
                         "kernels only implement the 1/sqrt(head_dim) softmax scale")


def _is_decode(kwargs, query_states):
    """One query token per sequence on the GPU: attention over every cached
    key (bounded by the window that _decode_window derives) is exactly what
    the decode kernel computes.  The reference also requires a
    ``past_key_values`` keyword (triton_gqa_decode_hf.py:236), which
    transformers 5.x no longer passes to attention functions, so its adapter
    never engages under ``generate``; this one does."""
    return query_states.shape[2] == 1 and query_states.is_cuda and query_states.shape[-1] in HEAD_DIMS


def custom_hf_decode_attention_forward(module, query_states, key_states, value_states, attention_mask, scaling: float,
                                       dropout: float = 0.0, **kwargs) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """HF attention-interface function: a decode step (q_len == 1 with a KV
    cache) runs the sm_100a kernel and returns ([B, Q_H, D], None), which the
    model reshapes to [B, 1, Q_H * D] as it does the reference's output
    (triton_gqa_decode_hf.py:218-258); anything else goes to transformers' SDPA."""
    bsz, q_heads, q_len, head_dim = query_states.shape
    if _is_decode(kwargs, query_states):
        _check_scaling(scaling, head_dim)
        q = query_states.squeeze(2)
        lens, starts = _decode_window(kwargs, bsz, q.device, attention_mask, key_states.shape[2])
        out = dense_decode(q, key_states, value_states, lens, starts,
                           s_aux=_module_sinks(module, q_heads, q.device))
        return out, None
    return _fallback(module, query_states, key_states, value_states, attention_mask, scaling, dropout, **kwargs)


def register_attention_interface(name: str = "fk_decode", fp8: bool = False, paged: bool = False) -> str:
    """Register the adapter with transformers' ``AttentionInterface`` so that
    ``attn_implementation=name`` selects it for any model (the reference's
    module-global patch of ``eager_attention_forward``,
    fskernels/engine/fs_inference_engine.py:12-13, only takes effect under
    "eager" in transformers 5.x).  ``paged=True`` registers the paged-cache
    adapter (``custom_paged_attention_forward``).  Returns the registered name."""
    from transformers import AttentionInterface
    if paged:
        from .paged_attn.paged_adapter import custom_paged_attention_forward as fn
    elif fp8:
        from .gqa_decode_hf_fp8 import custom_hf_decode_attention_forward_fp8 as fn
    else:
        fn = custom_hf_decode_attention_forward
    AttentionInterface.register(name, fn)
    return name
