"""Hugging Face attention adapter that decodes from a ``PagedKVCache``.

Drop-in for ``custom_paged_attention_forward`` of the reference's paged demo
(benchmarks/run_hf_triton_fp8_paged.py:18-61), with the cache bound through
``set_paged_attention_cache`` instead of the demo's module globals
``_DEMO_PAGED_CACHE`` / ``_DEMO_SEQ_IDS`` (:14-15).

A decode call (q_len == 1; the reference also asks for a ``past_key_values``
keyword, which transformers 5.x no longer passes) of layer
``module.layer_idx``:
  1. at layer 0, reserves the new token's slot of every bound sequence
     (``PagedKVCache.begin_step``: pages allocated on the host, one
     host-to-device copy of the new block-table entries);
  2. writes the token's K/V (the last position of ``key_states`` /
     ``value_states``) of all sequences with one ``paged_kv_append`` kernel
     (the reference loops over sequences with a ``.item()`` per token, :38-40);
  3. runs ``paged_flash_decode`` over the layer's pools (e4m3 pools use the
     cache's ``k_scale``/``v_scale``; sinks come from ``module.sinks``);
  4. at the last layer, commits the step (``end_step``).
Every layer of one step therefore sees the same lengths; the reference's
``append_kv`` advances a sequence's length once per layer call
(fskernels/paged_attn/paged_kv_cache.py:132), so its later layers attend
past the token just written.

Any other call (prefill) goes to transformers' SDPA attention, as the
reference routes it to eager attention (:55-60); when ``write_prefill`` is
set, the prompt's K/V of every bound sequence are also written into the
paged cache (the demo does that by hand after prefill, :107-117).

Returns ``(out [B, Q_H, 1, D], None)`` as the reference does (:50).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch

from ..gqa_decode_hf import _check_scaling, _fallback, _module_sinks
from .paged_decode import paged_flash_decode
from .paged_kv_cache import PAGE_SIZE, PagedKVCache


@dataclass
class _Binding:
    cache: Optional[PagedKVCache] = None
    seq_ids: List[int] = field(default_factory=list)
    write_prefill: bool = True
    lens: Optional[torch.Tensor] = None  # lengths of the step in progress (device)
    bt: Optional[torch.Tensor] = None    # block-table rows of the step in progress (device)


_BOUND = _Binding()


def set_paged_attention_cache(cache: Optional[PagedKVCache], seq_ids: List[int], write_prefill: bool = True) -> None:
    """Bind the cache and the batch's sequence ids (row b of the model's batch
    is sequence ``seq_ids[b]``).  ``cache=None`` unbinds."""
    _BOUND.cache = cache
    _BOUND.seq_ids = list(seq_ids)
    _BOUND.write_prefill = bool(write_prefill)
    _BOUND.lens = None
    _BOUND.bt = None


def get_paged_attention_cache() -> Tuple[Optional[PagedKVCache], List[int]]:
    return _BOUND.cache, list(_BOUND.seq_ids)


def custom_paged_attention_forward(module, query_states, key_states, value_states, attention_mask, scaling: float,
                                   dropout: float = 0.0, **kwargs) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    bsz, q_heads, q_len, head_dim = query_states.shape
    cache = _BOUND.cache
    layer = int(getattr(module, "layer_idx", 0) or 0)
    if cache is not None and q_len == 1 and query_states.is_cuda:
        _check_scaling(scaling, head_dim)
        if len(_BOUND.seq_ids) != bsz:
            raise ValueError(f"bound {len(_BOUND.seq_ids)} sequence ids for a batch of {bsz}")
        if layer == 0 or _BOUND.lens is None:
            _BOUND.bt, _, _BOUND.lens = cache.begin_step(_BOUND.seq_ids)
        cache.append_kv_batch(layer, key_states[:, :, -1], value_states[:, :, -1])
        e4m3 = cache.dtype == torch.float8_e4m3fn
        out = paged_flash_decode(query_states.squeeze(2), cache.k_pool[layer], cache.v_pool[layer],
                                 _BOUND.bt, _BOUND.lens, PAGE_SIZE,
                                 s_aux=_module_sinks(module, q_heads, query_states.device),
                                 scale_k=cache.k_scale if e4m3 else None, scale_v=cache.v_scale if e4m3 else None,
                                 out_dtype=query_states.dtype if e4m3 else None)
        if layer == cache.num_layers - 1:
            cache.end_step()
            _BOUND.lens = None
            _BOUND.bt = None
        return out.unsqueeze(2), None
    if cache is not None and _BOUND.write_prefill and q_len > 1 and len(_BOUND.seq_ids) == bsz:
        for b, sid in enumerate(_BOUND.seq_ids):
            cache.write_prefill(sid, layer, key_states[b], value_states[b])
    return _fallback(module, query_states, key_states, value_states, attention_mask, scaling, dropout, **kwargs)
