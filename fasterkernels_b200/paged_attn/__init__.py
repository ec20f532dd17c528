"""Paged KV cache and paged decode (mirrors fskernels/paged_attn/__init__.py:1-4)."""
from .paged_adapter import custom_paged_attention_forward, get_paged_attention_cache, set_paged_attention_cache
from .paged_append import paged_kv_append
from .paged_decode import paged_flash_decode
from .paged_kv_cache import PAGE_SIZE, PagedKVCache

__all__ = ["PagedKVCache", "PAGE_SIZE", "paged_flash_decode", "paged_kv_append", "custom_paged_attention_forward",
           "set_paged_attention_cache", "get_paged_attention_cache"]
