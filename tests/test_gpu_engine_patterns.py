"""Engine call patterns: a kernel that is not part of this library writes what
the decode reads immediately before the decode call, on the same stream.

These are the orderings a serving engine produces on every step:
  * the HF static cache's ``index_copy_`` of the new token's K/V into the
    dense cache (fskernels/engine/cuda_graph_runner.py:76-81), then attention;
  * ``paged_kv_append`` of the new token into its page, then paged decode
    (the batched form of benchmarks/run_hf_triton_fp8_paged.py:38-53);
  * a torch elementwise op (the RoPE position) writing ``q`` just before.
Each pattern runs 1000 steps eagerly and 1000 graph replays, the graph
built as CUDAGraphRunner builds it (cuda_graph_runner.py:172-237: static
``cache_position`` advanced by ``fill_`` between replays, inputs copied into
static buffers), and every step's output is checked against the CPU oracle.
The decode kernel is launched with programmatic stream serialisation; these
tests pin that it reads nothing before the preceding kernel's writes are
visible.
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
STEPS = 1000


@pytest.fixture(scope="module")
def dev():
    return torch.device("cuda", 0)


class _Module:
    """Stands in for an HF attention module (the adapters read only these)."""
    def __init__(self, layer_idx=0):
        self.layer_idx = layer_idx
        self.num_key_value_groups = 4


def _check_dense_steps(outs, qs, kc, vc, pos0, window=None, s_aux=None, tol=F16_TOL):
    """outs[i] must equal the oracle over cache rows [start, pos0 + i + 1)."""
    outs = outs.float().cpu().numpy()
    qs = qs.float().cpu().numpy()
    k = kc.float().cpu().numpy()
    v = vc.float().cpu().numpy()
    B = k.shape[0]
    sa = None if s_aux is None else s_aux.cpu().numpy()
    for i in range(outs.shape[0]):
        L = pos0 + i + 1
        starts = None if window is None else [max(0, L - window)] * B
        ref = O.decode_dense(qs[i], k, v, [L] * B, starts, s_aux=sa)
        np.testing.assert_allclose(outs[i], ref, err_msg=f"step {i}", **tol)


def _dense_setup(dev, B=2, QH=32, KVH=8, D=128, pos0=200, steps=STEPS, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    S = pos0 + steps
    kc = torch.zeros(B, KVH, S, D, device=dev, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    kc[:, :, :pos0] = torch.randn(B, KVH, pos0, D, generator=g, device=dev).half()
    vc[:, :, :pos0] = torch.randn(B, KVH, pos0, D, generator=g, device=dev).half()
    k_tok = torch.randn(steps, B, KVH, 1, D, generator=g, device=dev).half()
    v_tok = torch.randn(steps, B, KVH, 1, D, generator=g, device=dev).half()
    q_raw = torch.randn(steps, B, QH, D, generator=g, device=dev).half()
    return kc, vc, k_tok, v_tok, q_raw


def _rope_like(q_in, pos):
    """A torch op that writes q from the step's raw projection and position
    (a stand-in for RoPE: the value depends on the position tensor)."""
    return (q_in * (1.0 + (pos.to(torch.float32) % 7) * 0.125)).to(q_in.dtype)


def _q_expected(q_raw, pos0):
    pos = torch.arange(pos0, pos0 + q_raw.shape[0], device=q_raw.device).view(-1, 1, 1, 1)
    return (q_raw * (1.0 + (pos.to(torch.float32) % 7) * 0.125)).to(q_raw.dtype)


def test_dense_index_copy_then_decode_eager(dev):
    pos0 = 200
    kc, vc, k_tok, v_tok, q_raw = _dense_setup(dev, pos0=pos0)
    B, QH, D = q_raw.shape[1:]
    outs = torch.empty_like(q_raw)
    pos = torch.zeros(1, dtype=torch.long, device=dev)
    for i in range(STEPS):
        pos.fill_(pos0 + i)
        kc.index_copy_(2, pos, k_tok[i])
        vc.index_copy_(2, pos, v_tok[i])
        q = _rope_like(q_raw[i], pos)
        lens = (pos + 1).to(torch.int32).expand(B)
        fk.flash_decode_gqa_hf_dense_optimized(q, kc, vc, lens, out=outs[i])
    torch.cuda.synchronize()
    assert N.read_status(dev) == 0
    _check_dense_steps(outs, _q_expected(q_raw, pos0), kc, vc, pos0)


@pytest.mark.parametrize("window", [None, 96])
def test_dense_adapter_cuda_graph_runner_pattern(dev, window):
    # the adapter captured as CUDAGraphRunner.build captures a decode step:
    # cache update (index_copy_ at the static cache_position), q from a torch
    # op, attention through custom_hf_decode_attention_forward; replayed with
    # the position advanced by fill_ between replays
    pos0 = 200
    steps = STEPS if window is None else 64
    kc, vc, k_tok, v_tok, q_raw = _dense_setup(dev, pos0=pos0, steps=steps, seed=1)
    B, QH, D = q_raw.shape[1:]
    static_pos = torch.tensor([pos0], dtype=torch.long, device=dev)
    static_q = torch.zeros(B, QH, D, device=dev, dtype=torch.float16)
    static_k = torch.zeros(B, 8, 1, D, device=dev, dtype=torch.float16)
    static_v = torch.zeros_like(static_k)
    kwargs = dict(cache_position=static_pos, past_key_values=object())
    if window is not None:
        kwargs["sliding_window"] = window
    mod = _Module()

    def step():
        kc.index_copy_(2, static_pos, static_k)
        vc.index_copy_(2, static_pos, static_v)
        q = _rope_like(static_q, static_pos)
        out, _ = fk.custom_hf_decode_attention_forward(mod, q.unsqueeze(2), kc, vc, None, D ** -0.5, **kwargs)
        return out

    # one eager warm-up step at pos0 (the first replay rewrites it identically)
    static_q.copy_(q_raw[0])
    static_k.copy_(k_tok[0])
    static_v.copy_(v_tok[0])
    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = step()
    outs = torch.empty_like(q_raw)
    for i in range(steps):
        static_pos.fill_(pos0 + i)
        static_q.copy_(q_raw[i])
        static_k.copy_(k_tok[i])
        static_v.copy_(v_tok[i])
        graph.replay()
        outs[i].copy_(static_out)
    torch.cuda.synchronize()
    assert N.read_status(dev) == 0
    _check_dense_steps(outs, _q_expected(q_raw, pos0), kc, vc, pos0, window=window)


@pytest.mark.parametrize("graph", [False, True])
def test_paged_append_then_decode(dev, graph):
    # paged_kv_append writes each sequence's new token into its page right
    # before paged_flash_decode reads it; q comes from a torch op
    from fasterkernels_b200.paged_attn import PagedKVCache, paged_kv_append
    B, QH, KVH, D = 3, 32, 8, 128
    pos0 = [37, 200, 5]
    steps = STEPS
    maxlen = max(pos0) + steps
    mb = (maxlen + 15) // 16
    cache = PagedKVCache(num_layers=1, num_pages=B * mb + 8, max_seqs=B, max_blocks_per_seq=mb, num_kv_heads=KVH,
                         head_dim=D, dtype=torch.float16, device=str(dev))
    ids = [cache.allocate_sequence() for _ in range(B)]
    # reserve every page up front so the block table is static across steps
    g = torch.Generator(device=dev).manual_seed(5)
    hist_k = [torch.randn(maxlen, KVH, D, generator=g, device=dev).half() for _ in range(B)]
    hist_v = [torch.randn(maxlen, KVH, D, generator=g, device=dev).half() for _ in range(B)]
    for b, sid in enumerate(ids):
        cache.write_prefill(sid, 0, hist_k[b][: pos0[b]].transpose(0, 1), hist_v[b][: pos0[b]].transpose(0, 1),
                            reserve=maxlen)
    bt = cache.get_block_table_tensor(ids)
    q_raw = torch.randn(steps, B, QH, D, generator=g, device=dev).half()
    k_step = torch.stack([hist_k[b][pos0[b]:pos0[b] + steps] for b in range(B)], dim=1)  # [steps, B, KVH, D]
    v_step = torch.stack([hist_v[b][pos0[b]:pos0[b] + steps] for b in range(B)], dim=1)
    pos = torch.tensor(pos0, dtype=torch.int32, device=dev)
    static_q = torch.zeros(B, QH, D, device=dev, dtype=torch.float16)
    static_k = torch.zeros(B, KVH, D, device=dev, dtype=torch.float16)
    static_v = torch.zeros_like(static_k)
    out = torch.empty(B, QH, D, device=dev, dtype=torch.float16)
    scale = torch.tensor(0.75, device=dev, dtype=torch.float16)

    def step():
        paged_kv_append(static_k, static_v, cache.k_pool[0], cache.v_pool[0], bt, pos)
        q = static_q * scale
        fk.paged_flash_decode(q, cache.k_pool[0], cache.v_pool[0], bt, pos + 1, 16, out=out)

    outs = torch.empty_like(q_raw)
    if graph:
        step_pos = torch.tensor(pos0, dtype=torch.int32, device=dev)
        pos.copy_(step_pos)
        static_q.copy_(q_raw[0]); static_k.copy_(k_step[0]); static_v.copy_(v_step[0])
        step()  # eager warm-up at step 0 (rewritten identically by the first replay)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step()
        for i in range(steps):
            pos.copy_(step_pos + i)
            static_q.copy_(q_raw[i]); static_k.copy_(k_step[i]); static_v.copy_(v_step[i])
            gr.replay()
            outs[i].copy_(out)
    else:
        for i in range(steps):
            if i > 0:
                pos.add_(1)  # one more torch kernel writing what the decode reads
            static_q.copy_(q_raw[i]); static_k.copy_(k_step[i]); static_v.copy_(v_step[i])
            step()
            outs[i].copy_(out)
    torch.cuda.synchronize()
    assert N.read_status(dev) == 0
    o = outs.float().cpu().numpy()
    qe = (q_raw * scale).float().cpu().numpy()
    hk = [h.float().cpu().numpy() for h in hist_k]
    hv = [h.float().cpu().numpy() for h in hist_v]
    for i in range(steps):
        lens = [p + i + 1 for p in pos0]
        kk = np.concatenate([hk[b][: lens[b]] for b in range(B)])
        vv = np.concatenate([hv[b][: lens[b]] for b in range(B)])
        cu = np.concatenate([[0], np.cumsum(lens)])
        np.testing.assert_allclose(o[i], O.decode_varlen(qe[i], kk, vv, cu), err_msg=f"step {i}", **F16_TOL)
