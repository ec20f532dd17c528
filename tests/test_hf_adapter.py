"""HF attention-interface adapter: registration and the non-decode path on CPU."""
import torch

import fasterkernels_b200 as fk


class _Mod(torch.nn.Module):
    num_key_value_groups = 4
    is_causal = True


def test_register_attention_interface():
    from transformers import AttentionInterface
    name = fk.register_attention_interface("fk_decode_test")
    assert AttentionInterface()[name] is fk.custom_hf_decode_attention_forward
    name8 = fk.register_attention_interface("fk_decode_test_fp8", fp8=True)
    assert AttentionInterface()[name8] is fk.custom_hf_decode_attention_forward_fp8


def test_prefill_falls_back_to_sdpa_on_cpu():
    q = torch.randn(2, 8, 5, 128)
    k = torch.randn(2, 2, 5, 128)
    v = torch.randn(2, 2, 5, 128)
    out, w = fk.custom_hf_decode_attention_forward(_Mod(), q, k, v, None, 128 ** -0.5)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k.repeat_interleave(4, 1), v.repeat_interleave(4, 1),
                                                           is_causal=True)
    torch.testing.assert_close(out, ref.transpose(1, 2), atol=1e-5, rtol=1e-5)


def test_decode_window_from_mask_and_cache_position():
    from fasterkernels_b200.gqa_decode_hf import _decode_window
    mask = torch.zeros(2, 1, 1, 6, dtype=torch.bool)
    mask[0, ..., 2:] = True   # left padding of 2
    mask[1, ..., :] = True
    lens, starts = _decode_window({}, 2, "cpu", mask, 6)
    assert lens.tolist() == [6, 6] and starts.tolist() == [2, 0]
    add = torch.zeros(2, 1, 1, 6)
    add[0, ..., :3] = float("-inf")
    lens, starts = _decode_window({}, 2, "cpu", add, 6)
    assert lens.tolist() == [6, 6] and starts.tolist() == [3, 0]
    lens, starts = _decode_window({"cache_position": torch.tensor([9]), "sliding_window": 4}, 2, "cpu")
    assert lens.tolist() == [10, 10] and starts.tolist() == [6, 6]
    lens, starts = _decode_window({}, 3, "cpu", None, 7)
    assert lens.tolist() == [7, 7, 7] and starts is None
