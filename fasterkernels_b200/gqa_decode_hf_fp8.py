"""FP8 e4m3 GQA decode on the HF dense cache, and its attention adapter.

Drop-in for fskernels/triton/triton_gqa_decode_hf_fp8.py:
  * ``FP8_DTYPE``/``FP8_MAX`` (:9-10) and ``quantize_to_fp8`` (:13-16): per-tensor
    scale = amax / 448 (floored at 1e-12 / 448), values clamped to +-448.
  * ``set_num_splits_fp8`` (:159-161): recorded, accepted, not needed (the
    split schedule is planned on the device).
  * ``flash_decode_gqa_hf_fp8(q_fp8, k_cache_fp8, v_cache_fp8, cache_lens,
    scale_q, scale_k, scale_v, out_dtype)`` (:164-227).  Q may be e4m3 (times
    scale_q, like the reference) or float16/bfloat16 (scale_q ignored).  K/V
    are widened e4m3 -> f16 in registers; scale_k folds into the logit scale
    and scale_v into the output, so nothing is rounded to f16 after scaling.
    Optional keyword extras: ``s_aux`` sinks, ``start_k_offsets``, ``out``.
  * ``custom_hf_decode_attention_forward_fp8`` (:230-283).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .gqa_decode import HEAD_DIM
from .gqa_decode_hf import (_check_scaling, _decode_window, _fallback, _is_decode, _module_sinks,
                            custom_hf_decode_attention_forward, dense_decode)

FP8_DTYPE = torch.float8_e4m3fn
FP8_MAX = 448.0

_DECODE_NUM_SPLITS_FP8: int = 1


def set_num_splits_fp8(n: int) -> None:
    global _DECODE_NUM_SPLITS_FP8
    n = int(n)
    if n < 1:
        raise ValueError("num_splits must be >= 1")
    _DECODE_NUM_SPLITS_FP8 = n


def get_num_splits_fp8() -> int:
    return _DECODE_NUM_SPLITS_FP8


def quantize_to_fp8(x: torch.Tensor):
    """(x_fp8, scale) with scale = max|x| / 448 as a 0-dim float32 tensor on x's device."""
    xf = x.float()
    scale = xf.abs().max().clamp(min=1e-12) / FP8_MAX
    x_fp8 = (xf / scale).clamp(-FP8_MAX, FP8_MAX).to(FP8_DTYPE)
    return x_fp8, scale


def flash_decode_gqa_hf_fp8(q_fp8, k_cache_fp8, v_cache_fp8, cache_lens, scale_q, scale_k, scale_v, out_dtype,
                            *, s_aux=None, start_k_offsets=None, out=None):
    if k_cache_fp8.dtype != FP8_DTYPE or v_cache_fp8.dtype != FP8_DTYPE:
        raise TypeError("k_cache_fp8 and v_cache_fp8 must be float8_e4m3fn")
    if q_fp8.dtype not in (FP8_DTYPE, torch.float16, torch.bfloat16):
        raise TypeError("q must be float8_e4m3fn, float16 or bfloat16")
    if q_fp8.dtype == FP8_DTYPE and scale_q is None:
        raise ValueError("scale_q is required for an fp8 query")
    return dense_decode(q_fp8, k_cache_fp8, v_cache_fp8, cache_lens, start_k_offsets, s_aux=s_aux,
                        scale_q=scale_q, scale_k=scale_k, scale_v=scale_v, out_dtype=out_dtype, out=out)


def custom_hf_decode_attention_forward_fp8(module, query_states, key_states, value_states, attention_mask,
                                           scaling: float, dropout: float = 0.0,
                                           **kwargs) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """As the reference adapter (:230-283): quantise Q, K and V per call with
    per-tensor scales, then decode.  A cache that is already e4m3 (with
    ``module.k_scale``/``module.v_scale`` tensors) is used without re-quantising.
    e4m3 KV runs at head dim 128 only: a 16-bit cache of another head dim
    decodes in 16 bits (custom_hf_decode_attention_forward) instead."""
    bsz, q_heads, q_len, head_dim = query_states.shape
    if head_dim != HEAD_DIM and key_states.dtype != FP8_DTYPE:
        return custom_hf_decode_attention_forward(module, query_states, key_states, value_states, attention_mask,
                                                  scaling, dropout, **kwargs)
    if _is_decode(kwargs, query_states):
        _check_scaling(scaling, head_dim)
        out_dtype = query_states.dtype
        q = query_states.squeeze(2)
        lens, starts = _decode_window(kwargs, bsz, q.device, attention_mask, key_states.shape[2])
        q8, sq = quantize_to_fp8(q)
        if key_states.dtype == FP8_DTYPE:
            k8, sk = key_states, getattr(module, "k_scale")
            v8, sv = value_states, getattr(module, "v_scale")
        else:
            k8, sk = quantize_to_fp8(key_states)
            v8, sv = quantize_to_fp8(value_states)
        out = flash_decode_gqa_hf_fp8(q8, k8, v8, lens, sq, sk, sv, out_dtype, start_k_offsets=starts,
                                      s_aux=_module_sinks(module, q_heads, q.device))
        return out, None
    return _fallback(module, query_states, key_states, value_states, attention_mask, scaling, dropout, **kwargs)
