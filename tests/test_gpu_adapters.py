"""GPU tests of the Hugging Face attention adapters.

* ``custom_hf_decode_attention_forward_fp8`` at head dim 128, both forms of
  the reference adapter (fskernels/triton/triton_gqa_decode_hf_fp8.py:230-283):
  16-bit caches quantised per call, and an e4m3 cache read with the module's
  ``k_scale``/``v_scale``; each checked against the oracle on the dequantised
  tensors, eagerly and captured in a CUDA graph replayed with a static
  ``cache_position`` advanced by ``fill_`` (cuda_graph_runner.py:172-237).
* ``custom_paged_attention_forward`` (benchmarks/run_hf_triton_fp8_paged.py:18-61)
  over a multi-layer step loop, against the oracle per layer.
* A small random-weight Qwen3 model (no checkpoint: random init of the
  architecture) decoding through each registered adapter, logits compared
  with the same model under transformers' SDPA attention.
"""
import numpy as np
import pytest
import torch

import fasterkernels_b200 as fk
from fasterkernels_b200 import _native as N
from oracle import gqa_decode_oracle as O

pytestmark = pytest.mark.gpu
F16_TOL = dict(atol=2e-3, rtol=1e-2)
FP8_TOL = dict(atol=2e-2, rtol=0)


@pytest.fixture(scope="module")
def dev():
    return torch.device("cuda", 0)


class _Module:
    """Stands in for an HF attention module (the adapters and the SDPA
    fallback read only these attributes)."""
    is_causal = True

    def __init__(self, layer_idx=0, k_scale=None, v_scale=None, sinks=None, groups=4):
        self.layer_idx = layer_idx
        self.num_key_value_groups = groups
        if k_scale is not None:
            self.k_scale, self.v_scale = k_scale, v_scale
        if sinks is not None:
            self.sinks = sinks


def _deq(x8, s):
    return (x8.float() * s.float()).cpu().numpy()


def _fp8_case(dev, B=3, QH=32, KVH=8, S=900, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    qs = torch.randn(B, QH, 1, 128, generator=g, device=dev).half()
    ks = torch.randn(B, KVH, S, 128, generator=g, device=dev).half()
    vs = torch.randn(B, KVH, S, 128, generator=g, device=dev).half()
    return qs, ks, vs


@pytest.mark.parametrize("sinks", [False, True])
def test_fp8_adapter_d128_quantises_16bit_caches_per_call(dev, sinks):
    qs, ks, vs = _fp8_case(dev, seed=1)
    B, QH = qs.shape[:2]
    s_aux = torch.randn(QH, device=dev) if sinks else None
    pos = torch.tensor([700], device=dev)
    out, _ = fk.custom_hf_decode_attention_forward_fp8(_Module(sinks=s_aux), qs, ks, vs, None, 128 ** -0.5,
                                                       cache_position=pos)
    torch.cuda.synchronize()
    assert out.shape == (B, QH, 128) and out.dtype == torch.float16
    # the oracle on exactly what the kernel sees: Q, K and V quantised with
    # per-tensor scales (quantize_to_fp8, triton_gqa_decode_hf_fp8.py:13-16)
    q8, sq = fk.quantize_to_fp8(qs.squeeze(2))
    k8, sk = fk.quantize_to_fp8(ks)
    v8, sv = fk.quantize_to_fp8(vs)
    ref = O.decode_dense(_deq(q8, sq), _deq(k8, sk), _deq(v8, sv), [701] * B,
                         s_aux=None if s_aux is None else s_aux.cpu().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, **FP8_TOL)
    # and within the FP8 tolerance of the unquantised attention
    ref16 = O.decode_dense(qs.squeeze(2).float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                           [701] * B, s_aux=None if s_aux is None else s_aux.cpu().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), ref16, atol=6e-2, rtol=0)


def test_fp8_adapter_d128_e4m3_cache_with_module_scales(dev):
    qs, ks, vs = _fp8_case(dev, seed=2)
    B = qs.shape[0]
    k8, sk = fk.quantize_to_fp8(ks)
    v8, sv = fk.quantize_to_fp8(vs)
    mod = _Module(k_scale=sk, v_scale=sv)
    pos = torch.tensor([512], device=dev)
    out, _ = fk.custom_hf_decode_attention_forward_fp8(mod, qs, k8, v8, None, 128 ** -0.5, cache_position=pos,
                                                       sliding_window=300)
    torch.cuda.synchronize()
    q8, sq = fk.quantize_to_fp8(qs.squeeze(2))
    ref = O.decode_dense(_deq(q8, sq), _deq(k8, sk), _deq(v8, sv), [513] * B, [213] * B)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, **FP8_TOL)


@pytest.mark.parametrize("e4m3_cache", [False, True])
def test_fp8_adapter_cuda_graph_runner_pattern(dev, e4m3_cache):
    qs, ks, vs = _fp8_case(dev, B=2, S=600, seed=3)
    B, QH = qs.shape[:2]
    pos0 = 400
    k8, sk = fk.quantize_to_fp8(ks)
    v8, sv = fk.quantize_to_fp8(vs)
    kc, vc = (k8, v8) if e4m3_cache else (ks, vs)
    mod = _Module(k_scale=sk, v_scale=sv) if e4m3_cache else _Module()
    static_pos = torch.tensor([pos0], device=dev)
    static_q = qs.clone()

    def step():
        out, _ = fk.custom_hf_decode_attention_forward_fp8(mod, static_q, kc, vc, None, 128 ** -0.5,
                                                           cache_position=static_pos)
        return out

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = step()
    g = torch.Generator(device=dev).manual_seed(4)
    for r in range(4):
        p = pos0 + 37 * r
        static_pos.fill_(p)
        newq = torch.randn(qs.shape, generator=g, device=dev).half()
        static_q.copy_(newq)
        graph.replay()
        torch.cuda.synchronize()
        q8, sq = fk.quantize_to_fp8(newq.squeeze(2))
        ref = O.decode_dense(_deq(q8, sq), _deq(k8, sk), _deq(v8, sv), [p + 1] * B)
        np.testing.assert_allclose(static_out.float().cpu().numpy(), ref, err_msg=f"replay {r}", **FP8_TOL)
    assert N.read_status(dev) == 0


def test_adapters_refuse_a_non_default_scaling(dev):
    qs, ks, vs = _fp8_case(dev, B=1, S=32)
    pos = torch.tensor([31], device=dev)
    with pytest.raises(ValueError, match="scaling"):
        fk.custom_hf_decode_attention_forward(_Module(), qs, ks, vs, None, 0.5, cache_position=pos)
    with pytest.raises(ValueError, match="scaling"):
        fk.custom_hf_decode_attention_forward_fp8(_Module(), qs, ks, vs, None, 0.5, cache_position=pos)


@pytest.mark.parametrize("pool_dtype", [torch.float16, torch.float8_e4m3fn])
def test_paged_adapter_multi_layer_steps(dev, pool_dtype):
    from fasterkernels_b200.paged_attn import PagedKVCache, set_paged_attention_cache
    L, B, QH, KVH, D = 3, 2, 16, 4, 128
    cache = PagedKVCache(num_layers=L, num_pages=64, max_seqs=4, max_blocks_per_seq=16, num_kv_heads=KVH,
                         head_dim=D, dtype=pool_dtype, device=str(dev))
    if pool_dtype == torch.float8_e4m3fn:
        cache.set_fp8_scales(4.0 / 448, 4.0 / 448)
    ids = [cache.allocate_sequence(), cache.allocate_sequence()]
    set_paged_attention_cache(cache, ids)
    g = torch.Generator(device=dev).manual_seed(7)
    T0 = 21
    hist = {l: [torch.randn(B, KVH, T0, D, generator=g, device=dev).half(),
                torch.randn(B, KVH, T0, D, generator=g, device=dev).half()] for l in range(L)}
    try:
        # prefill: q_len > 1 goes to SDPA and writes the prompt into the pages
        for l in range(L):
            q = torch.randn(B, QH, T0, D, generator=g, device=dev).half()
            fk.custom_paged_attention_forward(_Module(l), q, hist[l][0], hist[l][1], None, D ** -0.5)
        assert [cache.seq_len(s) for s in ids] == [T0, T0]
        for step in range(20):
            for l in range(L):
                kn = torch.randn(B, KVH, 1, D, generator=g, device=dev).half()
                vn = torch.randn(B, KVH, 1, D, generator=g, device=dev).half()
                hist[l][0] = torch.cat([hist[l][0], kn], 2)
                hist[l][1] = torch.cat([hist[l][1], vn], 2)
                q = torch.randn(B, QH, 1, D, generator=g, device=dev).half()
                out, _ = fk.custom_paged_attention_forward(_Module(l), q, hist[l][0], hist[l][1], None, D ** -0.5)
                assert out.shape == (B, QH, 1, D)
                kk, vv = hist[l][0].float(), hist[l][1].float()
                if pool_dtype == torch.float8_e4m3fn:
                    kk = (kk / cache.k_scale).clamp(-448, 448).to(pool_dtype).float() * cache.k_scale
                    vv = (vv / cache.v_scale).clamp(-448, 448).to(pool_dtype).float() * cache.v_scale
                n = T0 + step + 1
                ref = O.decode_dense(q.squeeze(2).float().cpu().numpy(), kk.cpu().numpy(), vv.cpu().numpy(), [n] * B)
                tol = F16_TOL if pool_dtype == torch.float16 else FP8_TOL
                np.testing.assert_allclose(out.squeeze(2).float().cpu().numpy(), ref, err_msg=f"step {step} layer {l}",
                                           **tol)
            assert [cache.seq_len(s) for s in ids] == [T0 + step + 1] * 2  # one token per step, not per layer
    finally:
        set_paged_attention_cache(None, [])
    assert N.read_status(dev) == 0


def _tiny_qwen3(dev, dtype=torch.float16):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=4096)
    torch.manual_seed(0)
    return Qwen3ForCausalLM(cfg).to(device=dev, dtype=dtype).eval(), cfg


@pytest.mark.parametrize("impl", ["dense", "paged"])
def test_qwen3_random_weights_decode_matches_sdpa(dev, impl):
    from transformers import DynamicCache
    from fasterkernels_b200.paged_attn import PagedKVCache, set_paged_attention_cache
    model, cfg = _tiny_qwen3(dev)
    name = fk.register_attention_interface(f"fk_{impl}_qwen3_test", paged=(impl == "paged"))
    g = torch.Generator(device=dev).manual_seed(11)
    B, T0, steps = 3, 300, 12
    prompt = torch.randint(0, cfg.vocab_size, (B, T0), generator=g, device=dev)
    feed = torch.randint(0, cfg.vocab_size, (steps, B, 1), generator=g, device=dev)

    def run(attn):
        model.config._attn_implementation = attn
        cache = DynamicCache(config=cfg)
        logits = []
        with torch.no_grad():
            model(input_ids=prompt, past_key_values=cache, use_cache=True)
            for i in range(steps):
                o = model(input_ids=feed[i], past_key_values=cache, use_cache=True)
                logits.append(o.logits[:, -1].float())
        return torch.stack(logits)

    ref = run("sdpa")
    if impl == "paged":
        pc = PagedKVCache.from_config(cfg, num_pages=256, max_seqs=B, max_blocks_per_seq=64, device=str(dev),
                                      dtype=torch.float16)
        set_paged_attention_cache(pc, [pc.allocate_sequence() for _ in range(B)])
    try:
        got = run(name)
    finally:
        set_paged_attention_cache(None, [])
        model.config._attn_implementation = "sdpa"
    if impl == "paged":
        assert all(pc.seq_len(s) == T0 + steps for s in range(B))
    torch.testing.assert_close(got, ref, atol=3e-2, rtol=3e-2)
