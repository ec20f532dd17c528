"""The allocation-free varlen entry point, called through the C-ABI.

fk_flash_decode_gqa_varlen_noalloc serves callers that cannot allocate device
memory (a plugin inside a framework that owns all allocations, or a process
that forbids cudaMalloc once serving starts): its scratch is a fixed array
inside the library.  These tests check that two calls in a row match the
regular workspace entry point within the fp16 tolerance used by the other GPU
tests, and that a batch too large for the fixed scratch is refused with a
clear error.  The file name makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest
import torch

import fasterkernels_b200 as fk
from fasterkernels_b200 import _native as N
from fasterkernels_b200 import workloads as W

pytestmark = pytest.mark.gpu
F16_TOL = dict(atol=2e-3, rtol=1e-2)


def _bind():
    L = N.lib()
    f = L.fk_flash_decode_gqa_varlen_noalloc
    P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    f.restype = I
    f.argtypes = [P, P, P, P, P, P, I, I, I, I, LL, I, LL, LL, LL, LL, LL, LL, LL, LL, P]
    L.fk_noalloc_scratch_bytes.restype = ctypes.c_size_t
    L.fk_noalloc_scratch_bytes.argtypes = []
    return f


def _call(f, q, k, v, cu, s, out):
    dev = q.device
    return f(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(cu), N.ptr(s), N.ptr(out),
             q.shape[0], q.shape[1], k.shape[1], q.shape[2], k.shape[0], N.dtype_code(q.dtype),
             q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
             out.stride(0), out.stride(1), N.stream_of(dev))


def test_noalloc_matches_workspace_entry_on_two_calls():
    dev = torch.device("cuda", 0)
    f = _bind()
    for seed, lens in ((21, [3000, 17, 9000, 1, 0, 640]), (22, [12000, 5000, 33])):
        d = W.make_varlen(lens, 32, 8, torch.float16, dev, seed=seed, sinks=True)
        ref = fk.flash_decode_gqa_varlen(d["q"], d["k"], d["v"], d["cu_seqlens"], d["s_aux"])
        out = torch.full_like(d["q"], float("nan"))
        rc = _call(f, d["q"], d["k"], d["v"], d["cu_seqlens"], d["s_aux"], out)
        assert rc == 0, N.last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), **F16_TOL)


def test_noalloc_rejects_batches_beyond_its_scratch():
    dev = torch.device("cuda", 0)
    f = _bind()
    assert N.lib().fk_noalloc_scratch_bytes() == 8 << 20
    B = 4096  # 4096 * 8 items -> far more segments than the fixed scratch holds
    q = torch.zeros(B, 32, 128, device=dev, dtype=torch.float16)
    k = torch.zeros(B, 8, 128, device=dev, dtype=torch.float16)
    cu = torch.arange(B + 1, device=dev, dtype=torch.int32)
    out = torch.empty_like(q)
    rc = _call(f, q, k, k, cu, None, out)
    assert rc == 3 and "scratch" in N.last_error()
