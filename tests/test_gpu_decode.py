"""GPU parity tests: the sm_100a kernels (through the C-ABI via the Python
entry points) against the golden vectors and the CPU oracle.

Tolerances: fp16 output atol 2e-3 / rtol 1e-2 (fp32 accumulation); bf16
atol 1e-2 / rtol 2e-2 (bf16 P and V operands); FP8 KV atol 2e-2 against the
oracle on the dequantised KV; paged vs contiguous bit-identical.
"""
import time

import numpy as np
import pytest
import torch

import fasterkernels_b200 as fk
from fasterkernels_b200 import _native as N
from fasterkernels_b200 import workloads as W
from oracle import gqa_decode_oracle as O
from tests._golden import e4m3_to_float, load, paged_cases, varlen_cases

pytestmark = pytest.mark.gpu
F16_TOL = dict(atol=2e-3, rtol=1e-2)
BF16_TOL = dict(atol=1e-2, rtol=2e-2)
FP8_TOL = dict(atol=2e-2, rtol=0)


@pytest.fixture(scope="module")
def dev():
    return torch.device("cuda", 0)


def t(x, dev, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return x if dtype is None else x.to(dtype)


def close(out, ref, **tol):
    np.testing.assert_allclose(out.float().cpu().numpy(), np.asarray(ref, dtype=np.float64), **tol)


# ------------------------------------------------------------- golden cases
@pytest.mark.parametrize("name", varlen_cases())
def test_varlen_golden(dev, name):
    z = load(name)
    s = None if "s_aux" not in z else t(z["s_aux"], dev)
    out = fk.flash_decode_gqa_varlen(t(z["q"], dev), t(z["k"], dev), t(z["v"], dev), t(z["cu_seqlens"], dev), s)
    torch.cuda.synchronize()
    close(out, z["ref"], **F16_TOL)
    assert N.read_status(dev) == 0


@pytest.mark.parametrize("name", paged_cases())
def test_paged_golden_and_bit_identity(dev, name):
    z = load(name)
    q = t(z["q"], dev)
    kp, vp, bt, sl = t(z["k_pool"], dev), t(z["v_pool"], dev), t(z["block_table"], dev), t(z["seq_lens"], dev)
    out = fk.paged_flash_decode(q, kp, vp, bt, sl, 16)
    close(out, z["ref"], **F16_TOL)
    # same logical KV laid out contiguously -> bit-identical output
    lens = z["seq_lens"].tolist()
    ks = O.paged_to_dense(z["k_pool"], z["block_table"], z["seq_lens"])
    vs = O.paged_to_dense(z["v_pool"], z["block_table"], z["seq_lens"])
    kv = np.concatenate([x.transpose(1, 0, 2) for x in ks], 0)
    vv = np.concatenate([x.transpose(1, 0, 2) for x in vs], 0)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    out2 = fk.flash_decode_gqa_varlen(q, t(kv, dev), t(vv, dev), t(cu, dev))
    assert torch.equal(out, out2)


def test_dense_window_golden(dev):
    z = load("dense_g4_window")
    out = fk.flash_decode_gqa_hf_dense_optimized(t(z["q"], dev), t(z["k_cache"], dev), t(z["v_cache"], dev),
                                                 t(z["cache_lens"], dev), t(z["start_k_offsets"], dev))
    close(out, z["ref"], **F16_TOL)


def test_fp8_golden(dev):
    z = load("fp8_g4")
    k8 = t(z["k_fp8"], dev).view(torch.float8_e4m3fn)
    v8 = t(z["v_fp8"], dev).view(torch.float8_e4m3fn)
    sk = torch.tensor(float(z["scale_k"]), device=dev)
    sv = torch.tensor(float(z["scale_v"]), device=dev)
    lens = t(z["cache_lens"], dev)
    out = fk.flash_decode_gqa_hf_fp8(t(z["q"], dev), k8, v8, lens, None, sk, sv, torch.float16)
    close(out, z["ref"], **FP8_TOL)
    close(out, z["ref"], atol=3e-3, rtol=1e-2)  # fp16 Q, exact e4m3 widening: much tighter in practice
    q8 = t(z["q_fp8"], dev).view(torch.float8_e4m3fn)
    sq = torch.tensor(float(z["scale_q"]), device=dev)
    out8 = fk.flash_decode_gqa_hf_fp8(q8, k8, v8, lens, sq, sk, sv, torch.float16)
    close(out8, z["ref_q8"], **FP8_TOL)
    close(out8, z["ref_kernel"], **FP8_TOL)


# ------------------------------------------------------------- random cases
def _rand_case(dev, lens, qh, kvh, dtype, sinks, seed):
    d = W.make_varlen(lens, qh, kvh, torch.float32, dev, seed=seed, sinks=sinks)
    q, k, v = d["q"].to(dtype), d["k"].to(dtype), d["v"].to(dtype)
    return q, k, v, d["cu_seqlens"], d["s_aux"]


def _oracle(q, k, v, cu, s):
    return O.decode_varlen(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                           cu.cpu().numpy(), None if s is None else s.cpu().numpy())


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("sinks", [False, True])
def test_varlen_group_sizes(dev, G, sinks):
    lens = [1, 15, 16, 17, 63, 64, 65, 700, 0, 2049]
    q, k, v, cu, s = _rand_case(dev, lens, 4 * G, 4, torch.float16, sinks, seed=10 + G)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(out, _oracle(q, k, v, cu, s), **F16_TOL)


def test_varlen_bf16(dev):
    q, k, v, cu, s = _rand_case(dev, [5, 300, 4097, 33], 32, 8, torch.bfloat16, True, seed=3)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    assert out.dtype == torch.bfloat16
    close(out, _oracle(q, k, v, cu, s), **BF16_TOL)


def test_long_single_sequence_spans_many_ctas(dev):
    # one sequence over every CTA: exercises the multi-segment combine
    q, k, v, cu, s = _rand_case(dev, [70001], 32, 8, torch.float16, True, seed=4)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(out, _oracle(q, k, v, cu, s), **F16_TOL)


def test_workspace_counters_rearmed(dev):
    # every launch leaves the per-item arrival counters at zero
    q, k, v, cu, s = _rand_case(dev, [9000, 12000, 5], 32, 8, torch.float16, True, seed=12)
    for _ in range(3):
        fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    torch.cuda.synchronize()
    for ws in N.device_workspaces(dev):
        assert int(ws[256:256 + 4 * 3 * 8].view(torch.int32).abs().sum()) == 0


def test_concurrent_streams_have_separate_workspaces(dev):
    # decode calls on two streams run concurrently: each stream has its own
    # workspace, so split-item counters and partials never collide
    cases = [_rand_case(dev, [20000, 9000, 31000, 4000], 32, 8, torch.float16, True, seed=70 + i) for i in range(2)]
    refs = [fk.flash_decode_gqa_varlen(*c) for c in cases]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(dev) for _ in cases]
    for st in streams:
        st.wait_stream(torch.cuda.current_stream(dev))
    outs = [[], []]
    for _ in range(6):
        for i, (st, c) in enumerate(zip(streams, cases)):
            with torch.cuda.stream(st):
                outs[i].append(fk.flash_decode_gqa_varlen(*c))
    torch.cuda.synchronize()
    for i in range(2):
        for o in outs[i]:
            assert torch.equal(o, refs[i])
    assert len(N.device_workspaces(dev)) >= 3


def test_workspace_shared_across_shapes(dev):
    # launches of different (B, KV_H) on one workspace must not disturb each
    # other's arrival counters: small batch first, then a larger split batch
    for lens, qh, kvh in (([900, 40], 8, 2), ([6000] * 40, 32, 8), ([30, 7000, 3], 16, 4), ([6000] * 40, 32, 8)):
        q, k, v, cu, s = _rand_case(dev, lens, qh, kvh, torch.float16, True, seed=len(lens))
        out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
        b = len(lens) - 1
        lo, hi = int(cu[b]), int(cu[b + 1])
        ref = O.decode_varlen(q[b:b + 1].float().cpu().numpy(), k[lo:hi].float().cpu().numpy(),
                              v[lo:hi].float().cpu().numpy(), np.array([0, hi - lo]), s.cpu().numpy())
        close(out[b:b + 1], ref, **F16_TOL)


def test_many_short_sequences(dev):
    lens = [int(x) for x in torch.randint(0, 40, (700,), generator=torch.Generator().manual_seed(5))]
    q, k, v, cu, s = _rand_case(dev, lens, 16, 4, torch.float16, True, seed=5)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(out, _oracle(q, k, v, cu, s), **F16_TOL)


def test_empty_batch(dev):
    q = torch.empty(0, 32, 128, device=dev, dtype=torch.float16)
    k = torch.zeros(16, 8, 128, device=dev, dtype=torch.float16)
    cu = torch.zeros(1, device=dev, dtype=torch.int32)
    assert fk.flash_decode_gqa_varlen(q, k, k, cu).shape == (0, 32, 128)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_paged_random_bit_identical_to_varlen(dev, dtype):
    lens = [1, 16, 17, 250, 3000, 0, 64, 1023]
    q, k, v, cu, s = _rand_case(dev, lens, 32, 8, dtype, True, seed=6)
    kp, vp, bt = W.varlen_to_paged(k, v, lens, 1.25, seed=6)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    outp = fk.paged_flash_decode(q, kp, vp, bt, sl, 16, s_aux=s)
    outv = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    assert torch.equal(outp, outv)
    close(outp, _oracle(q, k, v, cu, s), **(F16_TOL if dtype == torch.float16 else BF16_TOL))


def test_dense_bit_identical_to_varlen(dev):
    lens = [100, 2000, 1]
    S = 2100
    q, k, v, cu, s = _rand_case(dev, lens, 32, 8, torch.float16, True, seed=7)
    kc = torch.zeros(3, 8, S, 128, device=dev, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    for b, L in enumerate(lens):
        kc[b, :, :L] = k[cu[b]:cu[b + 1]].transpose(0, 1)
        vc[b, :, :L] = v[cu[b]:cu[b + 1]].transpose(0, 1)
    outd = fk.gqa_decode_hf.dense_decode(q, kc, vc, torch.tensor(lens, device=dev, dtype=torch.int32), s_aux=s)
    outv = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    assert torch.equal(outd, outv)


def test_fp8_paged_sinks_vs_dense_and_oracle(dev):
    lens = [4000, 17, 1000, 2500]
    d = W.make_varlen(lens, 64, 8, torch.float32, dev, seed=8, sinks=True)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    q = d["q"].half()
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=8)
    kp, vp = kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    outp = fk.paged_flash_decode(q, kp, vp, bt, sl, 16, s_aux=d["s_aux"], scale_k=sk, scale_v=sv)
    kd = (k8.float() * sk).cpu().numpy()
    vd = (v8.float() * sv).cpu().numpy()
    ref = O.decode_varlen(q.float().cpu().numpy(), kd, vd, d["cu_seqlens"].cpu().numpy(), d["s_aux"].cpu().numpy())
    close(outp, ref, **FP8_TOL)
    close(outp, ref, atol=3e-3, rtol=1e-2)
    # dense cache with the same bytes -> bit-identical
    S = max(lens)
    kc = torch.zeros(4, 8, S, 128, device=dev, dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    cu = d["cu_seqlens"]
    for b, L in enumerate(lens):
        kc[b, :, :L] = k8.view(torch.uint8)[cu[b]:cu[b + 1]].transpose(0, 1)
        vc[b, :, :L] = v8.view(torch.uint8)[cu[b]:cu[b + 1]].transpose(0, 1)
    outd = fk.flash_decode_gqa_hf_fp8(q, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), sl, None, sk,
                                      sv, torch.float16, s_aux=d["s_aux"])
    assert torch.equal(outd, outp)


def test_bad_page_sets_status_and_masks(dev):
    lens = [40]
    q, k, v, cu, s = _rand_case(dev, lens, 32, 8, torch.float16, False, seed=9)
    kp, vp, bt = W.varlen_to_paged(k, v, lens, 1.0, seed=9)
    N.read_status(dev)
    bt_bad = bt.clone()
    bt_bad[0, 1] = 10_000_000  # out of the pool: page 1 (tokens 16..31) is skipped and masked
    out = fk.paged_flash_decode(q, kp, vp, bt_bad, torch.tensor(lens, device=dev, dtype=torch.int32), 16)
    torch.cuda.synchronize()
    assert N.read_status(dev) & N.FK_STATUS_BAD_PAGE
    keep = torch.cat([torch.arange(0, 16), torch.arange(32, 40)]).to(dev)
    cu2 = torch.tensor([0, 24], device=dev, dtype=torch.int32)
    ref = fk.flash_decode_gqa_varlen(q, k[keep].contiguous(), v[keep].contiguous(), cu2)
    close(out, ref.float().cpu().numpy(), atol=1e-3, rtol=1e-3)


def test_cuda_graph_capture_and_replay(dev):
    lens = [300, 5000, 77]
    q, k, v, cu, s = _rand_case(dev, lens, 32, 8, torch.float16, True, seed=11)
    out = torch.empty_like(q)
    fk.flash_decode_gqa_varlen(q, k, v, cu, s, out=out)  # warm-up sizes the workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fk.flash_decode_gqa_varlen(q, k, v, cu, s, out=out)
    q.copy_(torch.randn_like(q))
    cu.copy_(torch.tensor([0, 200, 5100, 5377], dtype=torch.int32, device=dev))  # new lengths, same graph
    g.replay()
    torch.cuda.synchronize()
    close(out, _oracle(q, k, v, cu, s), **F16_TOL)


def test_hf_adapter(dev):
    class M:
        num_key_value_heads = 8
    lens_pos = torch.tensor([900], device=dev)
    B, S = 2, 1024
    qs = torch.randn(B, 32, 1, 128, device=dev, dtype=torch.float16)
    ks = torch.randn(B, 8, S, 128, device=dev, dtype=torch.float16)
    vs = torch.randn(B, 8, S, 128, device=dev, dtype=torch.float16)
    out, w = fk.custom_hf_decode_attention_forward(M(), qs, ks, vs, None, 128 ** -0.5, past_key_values=object(),
                                                   cache_position=lens_pos)
    assert w is None and out.shape == (B, 32, 128)
    ref = O.decode_dense(qs.squeeze(2).float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                         [901, 901])
    close(out, ref, **F16_TOL)
    out_w, _ = fk.custom_hf_decode_attention_forward(M(), qs, ks, vs, None, 128 ** -0.5, past_key_values=object(),
                                                     cache_position=lens_pos, sliding_window=256)
    ref_w = O.decode_dense(qs.squeeze(2).float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                           [901, 901], [645, 645])
    close(out_w, ref_w, **F16_TOL)


def test_hf_adapters_head_dim_64(dev):
    # a head-dim-64 model through both HF adapters: the 16-bit kernel runs it,
    # the FP8 adapter included (e4m3 KV is served at head dim 128 only)
    class M:
        num_key_value_heads = 8
    lens_pos = torch.tensor([700], device=dev)
    B, S = 2, 1024
    qs = torch.randn(B, 64, 1, 64, device=dev, dtype=torch.bfloat16)
    ks = torch.randn(B, 8, S, 64, device=dev, dtype=torch.bfloat16)
    vs = torch.randn(B, 8, S, 64, device=dev, dtype=torch.bfloat16)
    ref = O.decode_dense(qs.squeeze(2).float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                         [701, 701])
    for fn in (fk.custom_hf_decode_attention_forward, fk.custom_hf_decode_attention_forward_fp8):
        out, w = fn(M(), qs, ks, vs, None, 64 ** -0.5, past_key_values=object(), cache_position=lens_pos)
        assert w is None and out.shape == (B, 64, 64)
        close(out, ref, **BF16_TOL)


# ------------------------------------------------- full benchmark sizes
def test_config2_full_size(dev):
    lens = W.config_lengths(2)
    assert sum(lens) == 377152
    d = W.make_varlen(lens, 32, 8, torch.float16, dev, seed=0, sinks=True)
    out = fk.flash_decode_gqa_varlen(d["q"], d["k"], d["v"], d["cu_seqlens"], d["s_aux"])
    cu = d["cu_seqlens"].cpu().numpy()
    # spot-check whole sequences against the oracle: the longest, the
    # shortest and six more spread over the batch
    picks = sorted({int(np.argmax(lens)), int(np.argmin(lens)), 0, 5, 11, 17, 24, 31})
    assert len(picks) >= 8
    for b in picks:
        lo, hi = cu[b], cu[b + 1]
        ref = O.decode_varlen(d["q"][b:b + 1].float().cpu().numpy(), d["k"][lo:hi].float().cpu().numpy(),
                              d["v"][lo:hi].float().cpu().numpy(), np.array([0, hi - lo]), d["s_aux"].cpu().numpy())
        close(out[b:b + 1], ref, **F16_TOL)
    # determinism: same inputs -> identical bits
    assert torch.equal(out, fk.flash_decode_gqa_varlen(d["q"], d["k"], d["v"], d["cu_seqlens"], d["s_aux"]))
    assert N.read_status(dev) == 0


def test_config3_full_size_paged_equals_varlen(dev):
    lens = W.config_lengths(3)
    d = W.make_varlen(lens, 32, 8, torch.float16, dev, seed=0, sinks=False)
    kp, vp, bt = W.varlen_to_paged(d["k"], d["v"], lens, 1.25, seed=0)
    assert kp.shape[0] == 21555
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    outp = fk.paged_flash_decode(d["q"], kp, vp, bt, sl, 16)
    outv = fk.flash_decode_gqa_varlen(d["q"], d["k"], d["v"], d["cu_seqlens"])
    assert torch.equal(outp, outv)
    cu = d["cu_seqlens"].cpu().numpy()
    picks = sorted({int(np.argmax(lens)), int(np.argmin(lens)), 0, 9, 21, 33, 47, 63})
    assert len(picks) >= 8
    for b in picks:
        lo, hi = cu[b], cu[b + 1]
        ref = O.decode_varlen(d["q"][b:b + 1].float().cpu().numpy(), d["k"][lo:hi].float().cpu().numpy(),
                              d["v"][lo:hi].float().cpu().numpy(), np.array([0, hi - lo]))
        close(outp[b:b + 1], ref, **F16_TOL)


def test_config4_full_size_fp8_paged_equals_dense(dev):
    lens = W.config_lengths(4)
    d = W.make_varlen(lens, 32, 8, torch.float16, dev, seed=0, sinks=True)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.0, seed=0)
    kp, vp = kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    outp = fk.paged_flash_decode(d["q"], kp, vp, bt, sl, 16, s_aux=d["s_aux"], scale_k=sk, scale_v=sv)
    kc = k8.view(16, 32768, 8, 128).transpose(1, 2)  # [B, KVH, S, D] strided view of the same bytes
    vc = v8.view(16, 32768, 8, 128).transpose(1, 2)
    outd = fk.flash_decode_gqa_hf_fp8(d["q"], kc, vc, sl, None, sk, sv, torch.float16, s_aux=d["s_aux"])
    assert torch.equal(outp, outd)
    for b in (0, 15):
        lo, hi = b * 32768, (b + 1) * 32768
        ref = O.decode_varlen(d["q"][b:b + 1].float().cpu().numpy(), (k8[lo:hi].float() * sk).cpu().numpy(),
                              (v8[lo:hi].float() * sv).cpu().numpy(), np.array([0, 32768]),
                              d["s_aux"].cpu().numpy())
        close(outp[b:b + 1], ref, **FP8_TOL)
    assert N.read_status(dev) == 0


def test_config5_full_size_fp8_paged_sinks(dev):
    # the multi-GPU benchmark configuration at its own size on one GPU:
    # B=128, Q_H=64, KV_H=8 (G=8), lengths log-U[4096, 131072], e4m3 paged
    # with sinks, pool x1.25 in a random page order
    spec = W.CONFIGS[5]
    lens = W.config_lengths(5)
    assert len(lens) == 128 and max(lens) <= 131072 and min(lens) >= 4096
    d = W.make_varlen(lens, spec.q_heads, spec.kv_heads, torch.float16, dev, seed=0, sinks=True)
    q, s_aux, cu_t = d["q"], d["s_aux"], d["cu_seqlens"]
    k8, sk = W.quantize_e4m3(d["k"])
    del d["k"]
    v8, sv = W.quantize_e4m3(d["v"])
    del d["v"]
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=0)
    kp, vp = kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    outp = fk.paged_flash_decode(q, kp, vp, bt, sl, 16, s_aux=s_aux, scale_k=sk, scale_v=sv)
    torch.cuda.synchronize()
    assert N.read_status(dev) == 0
    del kp, vp
    # the same logical KV on the HF dense cache: bit-identical
    cu = cu_t.cpu().numpy()
    S = max(lens)
    kc = torch.zeros(len(lens), spec.kv_heads, S, 128, dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    for b, L in enumerate(lens):
        kc[b, :, :L] = k8[cu[b]:cu[b + 1]].view(torch.uint8).transpose(0, 1)
        vc[b, :, :L] = v8[cu[b]:cu[b + 1]].view(torch.uint8).transpose(0, 1)
    outd = fk.flash_decode_gqa_hf_fp8(q, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), sl, None, sk, sv,
                                      torch.float16, s_aux=s_aux)
    torch.cuda.synchronize()
    assert torch.equal(outp, outd)
    assert N.read_status(dev) == 0
    del kc, vc
    # the oracle on the dequantised KV: longest, shortest and two median sequences
    order = np.argsort(lens)
    picks = [int(order[-1]), int(order[0]), int(order[len(lens) // 2 - 1]), int(order[len(lens) // 2])]
    for b in picks:
        lo, hi = cu[b], cu[b + 1]
        ref = O.decode_varlen(q[b:b + 1].float().cpu().numpy(), (k8[lo:hi].float() * sk).cpu().numpy(),
                              (v8[lo:hi].float() * sv).cpu().numpy(), np.array([0, hi - lo]), s_aux.cpu().numpy())
        close(outp[b:b + 1], ref, **FP8_TOL)


@pytest.mark.parametrize("kvh", [1, 3])
def test_odd_kv_heads_single_head_items(dev, kvh):
    # odd KV head counts run one KV head per work item; paged == varlen still holds
    lens = [1, 300, 2049, 17]
    q, k, v, cu, s = _rand_case(dev, lens, 4 * kvh, kvh, torch.float16, True, seed=30 + kvh)
    outv = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(outv, _oracle(q, k, v, cu, s), **F16_TOL)
    kp, vp, bt = W.varlen_to_paged(k, v, lens, 1.25, seed=kvh)
    outp = fk.paged_flash_decode(q, kp, vp, bt, torch.tensor(lens, dtype=torch.int32, device=dev), 16, s_aux=s)
    assert torch.equal(outp, outv)


def test_back_to_back_calls_overlapping_launches(dev):
    # consecutive decode kernels may overlap (programmatic dependent launch):
    # later calls that reuse the workspace and the output must not be
    # disturbed by, or disturb, the previous call
    cases = []
    for seed, lens in ((40, [9000, 3000, 12000]), (41, [50, 20000, 7]), (42, [4096] * 6)):
        cases.append(_rand_case(dev, lens, 32, 8, torch.float16, True, seed=seed))
    shared_out = torch.empty_like(cases[0][0])
    outs = []
    for rep in range(3):
        for i, (q, k, v, cu, s) in enumerate(cases):
            o = fk.flash_decode_gqa_varlen(q, k, v, cu, s, out=shared_out if i == 0 else None)
            outs.append((i, o))
    fk.flash_decode_gqa_varlen(*cases[0], out=shared_out)  # shared_out last written by case 0
    torch.cuda.synchronize()
    refs = [_oracle(*c) for c in cases]
    close(shared_out, refs[0], **F16_TOL)
    for i, o in outs:
        if i != 0:
            close(o, refs[i], **F16_TOL)
    assert N.read_status(dev) == 0


def test_chained_calls_output_fed_back_as_query(dev):
    # one call's output is the next call's query on the same stream: the
    # second launch must not start reading q before the first has written it
    q, k, v, cu, s = _rand_case(dev, [30000, 12000, 25000, 9000], 32, 8, torch.float16, True, seed=44)
    outs = [q]
    for _ in range(4):
        outs.append(fk.flash_decode_gqa_varlen(outs[-1], k, v, cu, s))
    torch.cuda.synchronize()
    for i in range(1, len(outs)):
        close(outs[i], _oracle(outs[i - 1], k, v, cu, s), **F16_TOL)
    # the same with a single buffer updated in place through out=
    x = q.clone()
    ref = q.clone()
    y = torch.empty_like(x)
    for _ in range(3):
        fk.flash_decode_gqa_varlen(x, k, v, cu, s, out=y)
        fk.flash_decode_gqa_varlen(y, k, v, cu, s, out=x)
    torch.cuda.synchronize()
    for _ in range(3):
        ref = torch.from_numpy(_oracle(torch.from_numpy(_oracle(ref, k, v, cu, s)).to(dev).half(), k, v, cu, s)).to(dev).half()
    close(x, ref.float().cpu().numpy(), atol=5e-3, rtol=2e-2)


@pytest.mark.parametrize("pool_dtype", [torch.float16, torch.bfloat16, torch.float8_e4m3fn])
def test_paged_kv_append_matches_torch(dev, pool_dtype):
    B, KVH, P = 5, 8, 40
    in_dtype = torch.bfloat16 if pool_dtype == torch.bfloat16 else torch.float16
    g = torch.Generator(device=dev).manual_seed(3)
    k_new = torch.randn(B, KVH, 128, generator=g, device=dev).to(in_dtype)
    v_new = torch.randn(B, KVH, 128, generator=g, device=dev).to(in_dtype)
    kp = torch.zeros(P, KVH, 16, 128, device=dev, dtype=torch.uint8 if pool_dtype == torch.float8_e4m3fn else pool_dtype)
    vp = torch.zeros_like(kp)
    if pool_dtype == torch.float8_e4m3fn:
        kp, vp = kp.view(pool_dtype), vp.view(pool_dtype)
    bt = torch.randperm(P, generator=torch.Generator().manual_seed(1))[:B * 4].view(B, 4).to(torch.int32).to(dev)
    pos = torch.tensor([0, 15, 16, 33, 63], dtype=torch.int32, device=dev)
    sk = torch.tensor(0.02, device=dev)
    sv = torch.tensor(0.03, device=dev)
    fk.paged_attn.paged_kv_append(k_new, v_new, kp, vp, bt, pos, scale_k=sk, scale_v=sv, increment=True)
    torch.cuda.synchronize()
    assert pos.tolist() == [1, 16, 17, 34, 64]
    for b, p0 in enumerate([0, 15, 16, 33, 63]):
        phys = int(bt[b, p0 // 16])
        if pool_dtype == torch.float8_e4m3fn:
            ek = (k_new[b].float() / sk).clamp(-448, 448).to(pool_dtype)
            ev = (v_new[b].float() / sv).clamp(-448, 448).to(pool_dtype)
            assert torch.equal(kp[phys, :, p0 % 16].view(torch.uint8), ek.view(torch.uint8))
            assert torch.equal(vp[phys, :, p0 % 16].view(torch.uint8), ev.view(torch.uint8))
        else:
            assert torch.equal(kp[phys, :, p0 % 16], k_new[b])
            assert torch.equal(vp[phys, :, p0 % 16], v_new[b])


def test_paged_cache_decode_loop_and_graph(dev):
    # a decode loop on PagedKVCache: prompt appended, then steps of
    # append (one kernel per layer) + decode, checked against the oracle; the
    # last step is captured in a CUDA graph and replayed with new inputs
    from fasterkernels_b200.paged_attn import PagedKVCache
    L, KVH, QH = 2, 8, 32
    cache = PagedKVCache(num_layers=L, num_pages=256, max_seqs=4, max_blocks_per_seq=64, num_kv_heads=KVH,
                         head_dim=128, dtype=torch.float16, device=str(dev))
    ids = [cache.allocate_sequence() for _ in range(3)]
    g = torch.Generator(device=dev).manual_seed(9)
    hist_k = {(l, s): [] for l in range(L) for s in ids}
    hist_v = {(l, s): [] for l in range(L) for s in ids}
    for step in range(40):
        bt, pos, lens = cache.begin_step(ids)
        for l in range(L):
            k = torch.randn(3, KVH, 128, generator=g, device=dev).half()
            v = torch.randn(3, KVH, 128, generator=g, device=dev).half()
            cache.append_kv_batch(l, k, v)
            for i, s in enumerate(ids):
                hist_k[(l, s)].append(k[i])
                hist_v[(l, s)].append(v[i])
        if step % 13 == 12:
            q = torch.randn(3, QH, 128, generator=g, device=dev).half()
            out = fk.paged_flash_decode(q, cache.k_pool[1], cache.v_pool[1], bt, lens, 16)
            kk = torch.cat([torch.stack(hist_k[(1, s)]) for s in ids]).float().cpu().numpy()
            vv = torch.cat([torch.stack(hist_v[(1, s)]) for s in ids]).float().cpu().numpy()
            cu = np.arange(0, 3 * (step + 2), step + 1)[:4]
            close(out, O.decode_varlen(q.float().cpu().numpy(), kk, vv, cu), **F16_TOL)
        cache.end_step()
    # graph-captured step: append + decode on fixed buffers
    bt, pos, lens = cache.begin_step(ids)
    k = torch.randn(3, KVH, 128, device=dev).half()
    v = torch.randn(3, KVH, 128, device=dev).half()
    q = torch.randn(3, QH, 128, device=dev).half()
    out = torch.empty_like(q)
    fk.paged_attn.paged_kv_append(k, v, cache.k_pool[0], cache.v_pool[0], bt, pos)
    fk.paged_flash_decode(q, cache.k_pool[0], cache.v_pool[0], bt, lens, 16, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fk.paged_attn.paged_kv_append(k, v, cache.k_pool[0], cache.v_pool[0], bt, pos)
        fk.paged_flash_decode(q, cache.k_pool[0], cache.v_pool[0], bt, lens, 16, out=out)
    k.copy_(torch.randn_like(k))
    q.copy_(torch.randn_like(q))
    graph.replay()
    torch.cuda.synchronize()
    for i, s in enumerate(ids):
        hist_k[(0, s)].append(k[i])
        hist_v[(0, s)].append(v[i])
    kk = torch.cat([torch.stack(hist_k[(0, s)]) for s in ids]).float().cpu().numpy()
    vv = torch.cat([torch.stack(hist_v[(0, s)]) for s in ids]).float().cpu().numpy()
    n = len(hist_k[(0, ids[0])])
    close(out, O.decode_varlen(q.float().cpu().numpy(), kk, vv, np.arange(0, 3 * n + 1, n)), **F16_TOL)


def test_hf_adapter_mask_derived_window(dev):
    # transformers 5.x style call: no cache_position, a padding mask
    class M:
        num_key_value_heads = 8
    B, S = 3, 700
    qs = torch.randn(B, 32, 1, 128, device=dev, dtype=torch.float16)
    ks = torch.randn(B, 8, S, 128, device=dev, dtype=torch.float16)
    vs = torch.randn(B, 8, S, 128, device=dev, dtype=torch.float16)
    mask = torch.ones(B, 1, 1, S, dtype=torch.bool, device=dev)
    mask[0, ..., :100] = False   # left padding
    mask[2, ..., :650] = False
    out, _ = fk.custom_hf_decode_attention_forward(M(), qs, ks, vs, mask, 128 ** -0.5, past_key_values=object())
    ref = O.decode_dense(qs.squeeze(2).float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                         [S, S, S], [100, 0, 650])
    close(out, ref, **F16_TOL)
    fk.register_attention_interface("fk_decode_gpu_test")


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_fp8_paged_group_sizes(dev, G):
    lens = [1, 31, 32, 33, 1500, 0, 4097]
    d = W.make_varlen(lens, 4 * G, 4, torch.float32, dev, seed=50 + G, sinks=True)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    q = d["q"].half()
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=G)
    out = fk.paged_flash_decode(q, kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn), bt,
                                torch.tensor(lens, dtype=torch.int32, device=dev), 16, s_aux=d["s_aux"],
                                scale_k=sk, scale_v=sv)
    ref = O.decode_varlen(q.float().cpu().numpy(), (k8.float() * sk).cpu().numpy(), (v8.float() * sv).cpu().numpy(),
                          d["cu_seqlens"].cpu().numpy(), d["s_aux"].cpu().numpy())
    close(out, ref, atol=3e-3, rtol=1e-2)


def test_fp8_dense_bf16_query_and_output(dev):
    B, S = 3, 3000
    lens = [2999, 1, 1800]
    g = torch.Generator(device=dev).manual_seed(60)
    q = torch.randn(B, 32, 128, generator=g, device=dev).bfloat16()
    k = torch.randn(B, 8, S, 128, generator=g, device=dev)
    v = torch.randn(B, 8, S, 128, generator=g, device=dev)
    k8, sk = W.quantize_e4m3(k)
    v8, sv = W.quantize_e4m3(v)
    out = fk.flash_decode_gqa_hf_fp8(q, k8, v8, torch.tensor(lens, dtype=torch.int32, device=dev), None, sk, sv,
                                     torch.bfloat16)
    assert out.dtype == torch.bfloat16
    ref = O.decode_dense(q.float().cpu().numpy(), (k8.float() * sk).cpu().numpy(), (v8.float() * sv).cpu().numpy(),
                         lens)
    close(out, ref, **BF16_TOL)


def test_dense_strided_cache_views(dev):
    # caches that are slices of larger allocations (HF StaticCache style) and
    # a query with a non-trivial batch stride
    big_k = torch.randn(4, 8, 5000, 128, device=dev, dtype=torch.float16)
    big_v = torch.randn(4, 8, 5000, 128, device=dev, dtype=torch.float16)
    kc, vc = big_k[1:3, :, :4096], big_v[1:3, :, :4096]
    qbig = torch.randn(2, 48, 128, device=dev, dtype=torch.float16)
    q = qbig[:, 8:40]
    lens = torch.tensor([4096, 2500], dtype=torch.int32, device=dev)
    starts = torch.tensor([0, 1000], dtype=torch.int32, device=dev)
    out = fk.flash_decode_gqa_hf_dense_optimized(q, kc, vc, lens, starts)
    ref = O.decode_dense(q.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(), [4096, 2500],
                         [0, 1000])
    close(out, ref, **F16_TOL)


def test_paged_strided_block_table(dev):
    lens = [100, 2000, 700]
    q, k, v, cu, s = _rand_case(dev, lens, 32, 8, torch.float16, True, seed=61)
    kp, vp, bt = W.varlen_to_paged(k, v, lens, 1.5, seed=61)
    wide = torch.full((3, 2 * bt.shape[1] + 5), -1, dtype=torch.int32, device=dev)
    wide[:, : bt.shape[1]] = bt
    out = fk.paged_flash_decode(q, kp, vp, wide[:, : bt.shape[1] + 3], torch.tensor(lens, dtype=torch.int32,
                                                                                     device=dev), 16, s_aux=s)
    assert torch.equal(out, fk.flash_decode_gqa_varlen(q, k, v, cu, s))


# ------------------------------------------------- groups of more than 8 heads
# The reference's Triton kernels take any group size (BLOCK_H pads it,
# fskernels/triton/triton_gqa_decode.py:132); here a group of more than 8
# query heads is split into items of at most 8 sharing the KV head.
@pytest.mark.parametrize("G,kvh", [(9, 4), (12, 8), (16, 8), (20, 2), (32, 2)])
@pytest.mark.parametrize("sinks", [False, True])
def test_varlen_large_groups(dev, G, kvh, sinks):
    lens = [1, 17, 64, 700, 0, 5000, 12345]
    q, k, v, cu, s = _rand_case(dev, lens, G * kvh, kvh, torch.float16, sinks, seed=80 + G)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(out, _oracle(q, k, v, cu, s), **F16_TOL)
    assert N.read_status(dev) == 0


def test_large_group_bf16_paged_matches_varlen_bitwise(dev):
    lens = [3000, 1, 16, 9000, 257]
    q, k, v, cu, s = _rand_case(dev, lens, 128, 8, torch.bfloat16, True, seed=91)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(out, _oracle(q, k, v, cu, s), **BF16_TOL)
    kp, vp, bt = W.varlen_to_paged(k, v, lens, 1.25, seed=3)
    outp = fk.paged_flash_decode(q, kp, vp, bt, torch.tensor(lens, dtype=torch.int32, device=dev), 16, s_aux=s)
    assert torch.equal(out, outp)


@pytest.mark.parametrize("G", [12, 16])
def test_fp8_large_groups_paged_and_dense(dev, G):
    lens = [1, 33, 1500, 0, 4097]
    kvh = 4
    d = W.make_varlen(lens, G * kvh, kvh, torch.float32, dev, seed=60 + G, sinks=True)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    q = d["q"].half()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=G)
    outp = fk.paged_flash_decode(q, kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn), bt, sl, 16,
                                 s_aux=d["s_aux"], scale_k=sk, scale_v=sv)
    ref = O.decode_varlen(q.float().cpu().numpy(), (k8.float() * sk).cpu().numpy(), (v8.float() * sv).cpu().numpy(),
                          d["cu_seqlens"].cpu().numpy(), d["s_aux"].cpu().numpy())
    close(outp, ref, atol=3e-3, rtol=1e-2)
    # the HF dense cache [B, KVH, S, D] with the same tokens
    S = max(lens)
    kc = torch.zeros(len(lens), kvh, S, 128, dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    cu = d["cu_seqlens"].tolist()
    for b, L in enumerate(lens):
        kc[b, :, :L] = k8.view(torch.uint8)[cu[b]:cu[b + 1]].transpose(0, 1)
        vc[b, :, :L] = v8.view(torch.uint8)[cu[b]:cu[b + 1]].transpose(0, 1)
    outd = fk.flash_decode_gqa_hf_fp8(q, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), sl, None, sk, sv,
                                      torch.float16, s_aux=d["s_aux"])
    assert torch.equal(outd, outp)


# ------------------------------------------------------------- head dim 64
# The reference's Triton kernels take any power-of-two head dim
# (triton_gqa_decode.py:136-152); 64 is served here for 16-bit KV.
def _rand_case_d(dev, lens, qh, kvh, dtype, sinks, seed, head_dim):
    d = W.make_varlen(lens, qh, kvh, torch.float32, dev, seed=seed, sinks=sinks, head_dim=head_dim)
    return d["q"].to(dtype), d["k"].to(dtype), d["v"].to(dtype), d["cu_seqlens"], d["s_aux"]


@pytest.mark.parametrize("G,kvh", [(1, 8), (4, 8), (8, 8), (8, 3), (16, 4)])
@pytest.mark.parametrize("sinks", [False, True])
def test_head_dim_64_varlen(dev, G, kvh, sinks):
    lens = [1, 15, 16, 17, 64, 700, 0, 9001]
    q, k, v, cu, s = _rand_case_d(dev, lens, G * kvh, kvh, torch.float16, sinks, 100 + G, 64)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    assert out.shape == q.shape
    close(out, _oracle(q, k, v, cu, s), **F16_TOL)
    assert N.read_status(dev) == 0


def test_head_dim_64_bf16_paged_dense_and_varlen_agree(dev):
    lens = [3000, 1, 0, 12000, 257, 64]
    B = len(lens)
    q, k, v, cu, s = _rand_case_d(dev, lens, 64, 8, torch.bfloat16, True, 7, 64)
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    close(out, _oracle(q, k, v, cu, s), **BF16_TOL)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    kp, vp, bt = W.varlen_to_paged(k, v, lens, 1.25, seed=5)
    outp = fk.paged_flash_decode(q, kp, vp, bt, sl, 16, s_aux=s)
    assert torch.equal(out, outp)
    S = max(lens)
    kc = torch.zeros(B, 8, S, 64, dtype=k.dtype, device=dev)
    vc = torch.zeros_like(kc)
    c = cu.tolist()
    for b, L in enumerate(lens):
        kc[b, :, :L] = k[c[b]:c[b + 1]].transpose(0, 1)
        vc[b, :, :L] = v[c[b]:c[b + 1]].transpose(0, 1)
    outd = fk.flash_decode_gqa_hf_dense_optimized(q, kc, vc, sl, s_aux=s)
    assert torch.equal(out, outd)
    # a sliding window on the dense cache
    st = torch.tensor([0, 0, 0, 11000, 200, 10], dtype=torch.int32, device=dev)
    outw = fk.flash_decode_gqa_hf_dense_optimized(q, kc, vc, sl, st, s_aux=s)
    ref = O.decode_dense(q.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                         lens, st.cpu().numpy(), s.cpu().numpy())
    close(outw, ref, **BF16_TOL)


def test_head_dim_64_append_then_decode(dev):
    B, KVH, P = 4, 8, 64
    g = torch.Generator(device=dev).manual_seed(9)
    k_new = torch.randn(B, KVH, 64, generator=g, device=dev).half()
    v_new = torch.randn(B, KVH, 64, generator=g, device=dev).half()
    kp = torch.zeros(P, KVH, 16, 64, device=dev, dtype=torch.float16)
    vp = torch.zeros_like(kp)
    bt = torch.randperm(P, generator=torch.Generator().manual_seed(2))[:B * 4].view(B, 4).to(torch.int32).to(dev)
    pos = torch.tensor([0, 15, 16, 40], dtype=torch.int32, device=dev)
    fk.paged_attn.paged_kv_append(k_new, v_new, kp, vp, bt, pos, increment=True)
    torch.cuda.synchronize()
    assert pos.tolist() == [1, 16, 17, 41]
    for b, p0 in enumerate([0, 15, 16, 40]):
        phys = int(bt[b, p0 // 16])
        assert torch.equal(kp[phys, :, p0 % 16], k_new[b])
        assert torch.equal(vp[phys, :, p0 % 16], v_new[b])
    with pytest.raises(ValueError):
        fk.paged_flash_decode(torch.zeros(B, 32, 64, device=dev, dtype=torch.float16), kp.view(torch.uint8)[..., :64]
                              .view(torch.float8_e4m3fn), kp.view(torch.uint8)[..., :64].view(torch.float8_e4m3fn),
                              bt, pos, 16)


def test_fp8_query_paged_raw_copy_matches_register_path(dev):
    # an e4m3 query with scale_q, as the reference's FP8 entry takes it: rows
    # aligned to 16 bytes are copied raw and converted by the consumers; an
    # unaligned strided view goes through the producer's registers.  Aligned
    # rows also let the kernel take four KV heads per work item (two for the
    # register path), so the two split the work differently and agree to
    # rounding.
    lens = [1, 33, 1500, 0, 4097, 777]
    d = W.make_varlen(lens, 32, 8, torch.float32, dev, seed=77, sinks=True)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    q8, sq = fk.quantize_to_fp8(d["q"])
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=4)
    kp, vp = kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    out = fk.paged_flash_decode(q8, kp, vp, bt, sl, 16, s_aux=d["s_aux"], scale_q=sq, scale_k=sk, scale_v=sv,
                                out_dtype=torch.float16)
    qbig = torch.zeros(len(lens), 32, 136, dtype=torch.uint8, device=dev)
    qbig[:, :, :128] = q8.view(torch.uint8)
    qv = qbig.view(torch.float8_e4m3fn)[:, :, :128]  # head stride 136 bytes: not 16-byte aligned
    out_v = fk.paged_flash_decode(qv, kp, vp, bt, sl, 16, s_aux=d["s_aux"], scale_q=sq, scale_k=sk, scale_v=sv,
                                  out_dtype=torch.float16)
    close(out_v, out.float().cpu().numpy(), atol=1e-3, rtol=1e-3)
    qd = (q8.float() * sq).half()
    ref = O.decode_varlen(qd.float().cpu().numpy(), (k8.float() * sk).cpu().numpy(), (v8.float() * sv).cpu().numpy(),
                          d["cu_seqlens"].cpu().numpy(), d["s_aux"].cpu().numpy())
    close(out, ref, atol=3e-3, rtol=1e-2)


def test_bounded_wait_runs_out_and_reports_timeout(dev):
    # Every mbarrier wait is bounded.  With the test hook each CTA's producer
    # publishes nothing for its first stage, so the consumers' wait on it runs
    # out (0.2 s here); the kernel returns with FK_STATUS_TIMEOUT instead of
    # hanging, the context stays usable, and the next call is correct.
    q, k, v, cu, s = _rand_case(dev, [3000, 50, 9000], 32, 8, torch.float16, True, seed=90)
    ref = _oracle(q, k, v, cu, s)
    fk.flash_decode_gqa_varlen(q, k, v, cu, s)  # workspace exists before the hook
    torch.cuda.synchronize()
    assert N.read_status(dev) == 0
    L = N.lib()
    assert L.fk_debug_configure(200_000_000, 1) == 0
    try:
        t0 = time.time()
        fk.flash_decode_gqa_varlen(q, k, v, cu, s)
        torch.cuda.synchronize()
        assert time.time() - t0 < 10.0
        assert N.read_status(dev) & N.FK_STATUS_TIMEOUT
    finally:
        assert L.fk_debug_configure(4_000_000_000, 0) == 0
    out = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
    torch.cuda.synchronize()
    close(out, ref, **F16_TOL)
    assert N.read_status(dev) == 0
    assert L.fk_debug_configure(10, 0) != 0  # out-of-range bound refused


# ------------------------------------------------- four KV heads per item
@pytest.mark.parametrize("G,kvh,qdt", [(5, 4, torch.float16), (6, 8, torch.float16), (8, 4, torch.bfloat16),
                                       (8, 8, torch.float8_e4m3fn)])
def test_fp8_four_head_items_paged_dense_and_oracle(dev, G, kvh, qdt):
    # e4m3 KV with kv_heads % 4 == 0 and groups of 5..8 query heads runs four
    # KV heads per work item (one TMA box per page and head quad); Q of
    # another type is converted by the consumers; paged == dense bits
    lens = [1, 15, 16, 17, 700, 0, 4097, 2049]
    d = W.make_varlen(lens, G * kvh, kvh, torch.float32, dev, seed=90 + G, sinks=True)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    if qdt == torch.float8_e4m3fn:
        q, sq = fk.quantize_to_fp8(d["q"])
        qref = (q.float() * sq).half().float()
    else:
        q, sq = d["q"].to(qdt), None
        qref = q.float()
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=G)
    outp = fk.paged_flash_decode(q, kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn), bt, sl, 16,
                                 s_aux=d["s_aux"], scale_q=sq, scale_k=sk, scale_v=sv, out_dtype=torch.float16)
    S = max(lens)
    kc = torch.zeros(len(lens), kvh, S, 128, dtype=torch.uint8, device=dev)
    vc = torch.zeros_like(kc)
    cu = d["cu_seqlens"].tolist()
    for b, L in enumerate(lens):
        kc[b, :, :L] = k8.view(torch.uint8)[cu[b]:cu[b + 1]].transpose(0, 1)
        vc[b, :, :L] = v8.view(torch.uint8)[cu[b]:cu[b + 1]].transpose(0, 1)
    outd = fk.flash_decode_gqa_hf_fp8(q, kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), sl, sq, sk, sv,
                                      torch.float16, s_aux=d["s_aux"])
    torch.cuda.synchronize()
    assert torch.equal(outd, outp)
    ref = O.decode_varlen(qref.cpu().numpy(), (k8.float() * sk).cpu().numpy(), (v8.float() * sv).cpu().numpy(),
                          d["cu_seqlens"].cpu().numpy(), d["s_aux"].cpu().numpy())
    close(outp, ref, atol=3e-3 if qdt == torch.float16 else 1e-2, rtol=1e-2)
    assert N.read_status(dev) == 0


def test_fp8_four_head_items_bad_pages(dev):
    lens = [40, 300]
    d = W.make_varlen(lens, 64, 8, torch.float32, dev, seed=95, sinks=False)
    k8, sk = W.quantize_e4m3(d["k"])
    v8, sv = W.quantize_e4m3(d["v"])
    kp, vp, bt = W.varlen_to_paged(k8.view(torch.uint8), v8.view(torch.uint8), lens, 1.25, seed=3)
    N.read_status(dev)
    bt = bt.clone()
    bt[1, 5] = kp.shape[0] + 7  # tokens 80..95 of sequence 1: outside the pool
    out = fk.paged_flash_decode(d["q"].half(), kp.view(torch.float8_e4m3fn), vp.view(torch.float8_e4m3fn), bt,
                                torch.tensor(lens, dtype=torch.int32, device=dev), 16, scale_k=sk, scale_v=sv)
    torch.cuda.synchronize()
    assert N.read_status(dev) & N.FK_STATUS_BAD_PAGE
    keep = np.r_[0:80, 96:300]
    k1 = (k8.float() * sk)[40:340][keep].cpu().numpy()
    v1 = (v8.float() * sv)[40:340][keep].cpu().numpy()
    ref = O.decode_varlen(d["q"][1:2].half().float().cpu().numpy(), k1, v1, np.array([0, len(keep)]))
    close(out[1:2], ref, atol=3e-3, rtol=1e-2)
