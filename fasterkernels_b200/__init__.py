"""fasterkernels_b200 -- B200 (sm_100a) GQA decode attention.

Entry points mirror coder0143/fasterkernels' decode API; the work runs in
hand-written sm_100a CUDA kernels behind the C-ABI of include/fk_decode.h.
"""
from ._native import read_status
from .gqa_decode import flash_decode_gqa_varlen
from .gqa_decode_hf import (custom_hf_decode_attention_forward, flash_decode_gqa_hf_dense_optimized,
                            get_num_splits, register_attention_interface, set_num_splits)
from .gqa_decode_hf_fp8 import (FP8_DTYPE, FP8_MAX, custom_hf_decode_attention_forward_fp8,
                                flash_decode_gqa_hf_fp8, get_num_splits_fp8, quantize_to_fp8, set_num_splits_fp8)
from .paged_attn import (PAGE_SIZE, PagedKVCache, custom_paged_attention_forward, paged_flash_decode,
                         set_paged_attention_cache)

__version__ = "0.1.0"

__all__ = [
    "flash_decode_gqa_varlen", "flash_decode_gqa_hf_dense_optimized", "custom_hf_decode_attention_forward",
    "set_num_splits", "get_num_splits", "flash_decode_gqa_hf_fp8", "custom_hf_decode_attention_forward_fp8",
    "quantize_to_fp8", "set_num_splits_fp8", "get_num_splits_fp8", "FP8_DTYPE", "FP8_MAX", "paged_flash_decode",
    "PagedKVCache", "PAGE_SIZE", "custom_paged_attention_forward", "set_paged_attention_cache", "read_status", "register_attention_interface",
]
