"""torch.compile traces through the decode entry points (registered as
torch.library custom ops) with fullgraph=True, i.e. without a graph break,
and the compiled results equal the eager ones bit for bit."""
import pytest
import torch

import fasterkernels_b200 as fk
from fasterkernels_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    return torch.device("cuda", 0)


def test_compile_fullgraph_varlen_and_paged(dev):
    torch._dynamo.reset()
    lens = [700, 33, 4097, 16]
    d = W.make_varlen(lens, 32, 8, torch.float16, dev, seed=3, sinks=True)
    kp, vp, bt = W.varlen_to_paged(d["k"], d["v"], lens, 1.25, seed=3)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)

    def step(q, k, v, cu, s, kp, vp, bt, sl):
        x = q * 0.5  # ops around the custom ops are compiled too (exact in fp16)
        a = fk.flash_decode_gqa_varlen(x, k, v, cu, s)
        b = fk.paged_flash_decode(x, kp, vp, bt, sl, 16, s_aux=s)
        return a, b, a + 1.0

    args = (d["q"], d["k"], d["v"], d["cu_seqlens"], d["s_aux"], kp, vp, bt, sl)
    ea, eb, ec = step(*args)
    ca, cb, cc = torch.compile(step, fullgraph=True)(*args)
    torch.cuda.synchronize()
    assert torch.equal(ea, ca) and torch.equal(eb, cb) and torch.equal(ec, cc)
    assert torch.equal(ea, eb)  # paged == varlen bits


def test_compile_fullgraph_dense_fp8_and_append(dev):
    torch._dynamo.reset()
    B, KVH, S = 3, 8, 600
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(B, 32, 128, generator=g, device=dev).half()
    kc = torch.randn(B, KVH, S, 128, generator=g, device=dev).half()
    vc = torch.randn(B, KVH, S, 128, generator=g, device=dev).half()
    k8, sk = fk.quantize_to_fp8(kc)
    v8, sv = fk.quantize_to_fp8(vc)
    lens = torch.tensor([600, 1, 333], dtype=torch.int32, device=dev)

    def step(q, kc, vc, k8, v8, lens):
        a = fk.flash_decode_gqa_hf_dense_optimized(q, kc, vc, lens)
        b = fk.flash_decode_gqa_hf_fp8(q, k8, v8, lens, None, sk, sv, torch.float16)
        return a, b

    ea, eb = step(q, kc, vc, k8, v8, lens)
    ca, cb = torch.compile(step, fullgraph=True)(q, kc, vc, k8, v8, lens)
    torch.cuda.synchronize()
    assert torch.equal(ea, ca) and torch.equal(eb, cb)

    # paged append (mutates the pools and the positions) inside a compiled step
    from fasterkernels_b200.paged_attn import paged_kv_append
    P = 8
    kp = torch.zeros(P, KVH, 16, 128, device=dev, dtype=torch.float16)
    vp = torch.zeros_like(kp)
    bt = torch.arange(B * 2, device=dev, dtype=torch.int32).view(B, 2) % P
    pos = torch.tensor([0, 5, 17], dtype=torch.int32, device=dev)
    kn = torch.randn(B, KVH, 128, generator=g, device=dev).half()
    vn = torch.randn(B, KVH, 128, generator=g, device=dev).half()

    def app(kn, vn, kp, vp, bt, pos):
        paged_kv_append(kn, vn, kp, vp, bt, pos, increment=True)
        return fk.paged_flash_decode(q, kp, vp, bt, pos, 16)

    kp2, vp2, pos2 = kp.clone(), vp.clone(), pos.clone()
    e = app(kn, vn, kp, vp, bt, pos)
    c = torch.compile(app, fullgraph=True)(kn, vn, kp2, vp2, bt, pos2)
    torch.cuda.synchronize()
    assert torch.equal(kp, kp2) and torch.equal(vp, vp2) and torch.equal(pos, pos2)
    assert pos.tolist() == [1, 6, 18]
    assert torch.equal(e, c)
