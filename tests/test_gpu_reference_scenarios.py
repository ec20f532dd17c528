"""The reference's own decode tests, restated: the same scenarios (shapes,
length draws, sink scale, page scatter, FP8 quantisation) through this
library's entry points, held to the reference's tolerance atol = rtol = 1e-3
against the attention oracle.

  tests/test_cuda_fd_gqa.py:38-69       native varlen, positional ``sink``
  tests/test_triton_fd_gqa.py:40-66     Triton varlen (same scenario)
  tests/test_tilelang_fd_gqa.py:40-69   TileLang varlen (same scenario)
  tests/test_triton_paged_gqa_decode.py:41-97  paged, scattered pages
  tests/test_triton_gqa_decode_fp8.py:34-74    FP8 dense, short and split-KV

Inputs are drawn from seeded CPU generators (the reference draws on the
device), so the values differ while the distributions match.
"""
import numpy as np
import pytest
import torch

import fasterkernels_b200 as fk
from fasterkernels_b200 import cuda_fd_gqa
from fasterkernels_b200 import workloads as W
from oracle import gqa_decode_oracle as O

pytestmark = pytest.mark.gpu
REF_TOL = dict(atol=1e-3, rtol=1e-3)


# bf16 keeps 8 significant bits: one rounding step of an output of 0.25 is
# already 2e-3, above the reference's 1e-3, so bf16 outputs are held to one
# bf16 step relative (2^-8) on top of the reference's absolute 1e-3.
BF16_STEP_TOL = dict(atol=1e-3, rtol=2.0 ** -8)


def _close(out, ref):
    tol = BF16_STEP_TOL if out.dtype == torch.bfloat16 else REF_TOL
    torch.testing.assert_close(out.float().cpu(), torch.as_tensor(np.asarray(ref), dtype=torch.float32), **tol)


@pytest.mark.parametrize("entry", ["triton", "cuda", "tilelang"])
def test_varlen_scenario(entry):
    dev = torch.device("cuda", 0)
    B, QH, KVH, MAX_S, D = 4, 32, 8, 4096, 128
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(MAX_S // 4, MAX_S + 1, (B,), generator=g)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0).to(torch.int32)
    T = int(cu[-1])
    q = torch.randn(B, QH, D, generator=g).half()
    k = torch.randn(T, KVH, D, generator=g).half()
    v = torch.randn(T, KVH, D, generator=g).half()
    sink = (torch.randn(QH, generator=g) * 0.1).float()
    args = (q.to(dev), k.to(dev), v.to(dev), cu.to(dev))
    if entry == "cuda":
        out = cuda_fd_gqa.flash_decode_gqa_varlen(*args, sink.to(dev))  # positional sink, as cuda_fd_gqa.py:14
    else:
        out = fk.flash_decode_gqa_varlen(*args, s_aux=sink.to(dev))
    torch.cuda.synchronize()
    _close(out, O.decode_varlen(q.numpy(), k.numpy(), v.numpy(), cu.numpy(), sink.numpy()))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])  # as test_triton_paged_gqa_decode.py:100-102
def test_paged_scenario(dtype):
    dev = torch.device("cuda", 0)
    B, QH, KVH, D, PS = 4, 32, 8, 128, 16
    lens = [64, 512, 1024, 250]
    g = torch.Generator().manual_seed(42)
    q = torch.randn(B, QH, D, generator=g).to(dtype)
    npages = [(L + PS - 1) // PS for L in lens]
    P = sum(npages) + 10  # spare pages, as the reference allocates
    k_pool = torch.zeros(P, KVH, PS, D, dtype=dtype)
    v_pool = torch.zeros_like(k_pool)
    perm = torch.randperm(P, generator=g)
    bt = torch.full((B, max(npages)), -1, dtype=torch.int32)
    i = 0
    for b, L in enumerate(lens):
        for pg in range(npages[b]):
            phys = int(perm[i])
            i += 1
            bt[b, pg] = phys
            n = min(PS, L - pg * PS)
            k_pool[phys, :, :n] = torch.randn(KVH, n, D, generator=g).to(dtype)
            v_pool[phys, :, :n] = torch.randn(KVH, n, D, generator=g).to(dtype)
    sl = torch.tensor(lens, dtype=torch.int32)
    out = fk.paged_flash_decode(q.to(dev), k_pool.to(dev), v_pool.to(dev), bt.to(dev), sl.to(dev), PS)
    torch.cuda.synchronize()
    _close(out, O.decode_paged(q.float().numpy(), k_pool.float().numpy(), v_pool.float().numpy(), bt.numpy(), lens))


def test_fp8_scenario():
    dev = torch.device("cuda", 0)
    B, QH, KVH, MAX_S, D = 4, 32, 8, 2048, 128
    g = torch.Generator().manual_seed(42)
    q = torch.randn(B, QH, D, generator=g).half()
    k = torch.randn(B, KVH, MAX_S, D, generator=g).half()
    v = torch.randn(B, KVH, MAX_S, D, generator=g).half()
    lens = torch.randint(MAX_S // 4, MAX_S + 1, (B,), generator=g).to(torch.int32)
    q8, sq = fk.quantize_to_fp8(q.float().to(dev))
    k8, sk = fk.quantize_to_fp8(k.float().to(dev))
    v8, sv = fk.quantize_to_fp8(v.float().to(dev))
    fk.set_num_splits_fp8(1)
    out = fk.flash_decode_gqa_hf_fp8(q8, k8, v8, lens.to(dev), sq, sk, sv, torch.float16)
    torch.cuda.synchronize()
    qd = (q8.float() * sq).half().float().cpu().numpy()  # the reference's ref on dequantised fp16 inputs
    kd = (k8.float() * sk).half().float().cpu().numpy()
    vd = (v8.float() * sv).half().float().cpu().numpy()
    _close(out, O.decode_dense(qd, kd, vd, lens.tolist()))
    # the split-KV case: 5000 of 6000 cache rows, num_splits 8
    kl = torch.randn(B, KVH, 6000, D, generator=g).half()
    vl = torch.randn(B, KVH, 6000, D, generator=g).half()
    kl8, skl = fk.quantize_to_fp8(kl.float().to(dev))
    vl8, svl = fk.quantize_to_fp8(vl.float().to(dev))
    fk.set_num_splits_fp8(8)
    ll = torch.full((B,), 5000, dtype=torch.int32, device=dev)
    out_l = fk.flash_decode_gqa_hf_fp8(q8, kl8, vl8, ll, sq, skl, svl, torch.float16)
    torch.cuda.synchronize()
    kdl = (kl8.float() * skl).half().float().cpu().numpy()
    vdl = (vl8.float() * svl).half().float().cpu().numpy()
    _close(out_l, O.decode_dense(qd, kdl, vdl, [5000] * B))
    fk.set_num_splits_fp8(1)
