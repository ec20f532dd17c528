"""The allocation-free varlen entry point, called through the C-ABI.

fk_flash_decode_gqa_varlen_noalloc serves callers that cannot allocate device
memory (a plugin inside a framework that owns all allocations, or a process
that forbids cudaMalloc once serving starts): its scratch is a fixed array
inside the library.  It runs the same plan on the same kernel as the
workspace entry point, so the tests require identical bits from the two and
check both against the CPU oracle at the fp16/bf16 tolerances of the other GPU
tests; they also check the size limit stated in include/fk_decode.h and that
a timed-out call is reported by fk_noalloc_read_status.  The file name makes
pytest collect it last.
"""
import ctypes

import numpy as np
import pytest
import torch

import fasterkernels_b200 as fk
from fasterkernels_b200 import _native as N
from fasterkernels_b200 import workloads as W
from oracle import gqa_decode_oracle as O

pytestmark = pytest.mark.gpu
TOL = {torch.float16: dict(atol=2e-3, rtol=1e-2), torch.bfloat16: dict(atol=1e-2, rtol=2e-2)}
SEG_BYTES = 4 + 16 * 8 + 16 * 128 * 4  # scratch bytes per segment record


def _bind():
    L = N.lib()
    f = L.fk_flash_decode_gqa_varlen_noalloc
    P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    f.restype = I
    f.argtypes = [P, P, P, P, P, P, I, I, I, I, LL, I, LL, LL, LL, LL, LL, LL, LL, LL, P]
    L.fk_noalloc_scratch_bytes.restype = ctypes.c_size_t
    L.fk_noalloc_scratch_bytes.argtypes = []
    L.fk_noalloc_read_status.restype = I
    L.fk_noalloc_read_status.argtypes = [I, ctypes.POINTER(I), I]
    return f


def _call(f, q, k, v, cu, s, out):
    dev = q.device
    return f(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(cu), N.ptr(s), N.ptr(out),
             q.shape[0], q.shape[1], k.shape[1], q.shape[2], k.shape[0], N.dtype_code(q.dtype),
             q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
             out.stride(0), out.stride(1), N.stream_of(dev))


def _status(dev, clear=1):
    st = ctypes.c_int(-1)
    assert N.lib().fk_noalloc_read_status(dev.index, ctypes.byref(st), clear) == 0, N.last_error()
    return st.value


def _case(dev, lens, qh, kvh, dtype, hd, seed):
    d = W.make_varlen(lens, qh, kvh, torch.float32, dev, seed=seed, sinks=True, head_dim=hd)
    return d["q"].to(dtype), d["k"].to(dtype), d["v"].to(dtype), d["cu_seqlens"], d["s_aux"]


def _oracle(q, k, v, cu, s):
    return O.decode_varlen(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                           cu.cpu().numpy(), s.cpu().numpy())


@pytest.mark.parametrize("dtype,hd,qh,kvh", [(torch.float16, 128, 32, 8), (torch.bfloat16, 128, 32, 8),
                                             (torch.float16, 64, 64, 8), (torch.float16, 128, 64, 4)])
def test_noalloc_matches_workspace_entry_on_two_calls(dtype, hd, qh, kvh):
    dev = torch.device("cuda", 0)
    f = _bind()
    cases = [_case(dev, [3000, 17, 9000, 1, 0, 640], qh, kvh, dtype, hd, seed=21),
             _case(dev, [12000, 5000, 33], qh, kvh, dtype, hd, seed=22)]
    outs = []
    # two allocation-free calls in a row, of different batch sizes
    for q, k, v, cu, s in cases:
        out = torch.full_like(q, float("nan"))
        rc = _call(f, q, k, v, cu, s, out)
        assert rc == 0, N.last_error()
        outs.append(out)
    torch.cuda.synchronize()
    assert _status(dev) == 0
    for (q, k, v, cu, s), out in zip(cases, outs):
        ref = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), "allocation-free and workspace entry points differ"
        np.testing.assert_allclose(out.float().cpu().numpy(), _oracle(q, k, v, cu, s), **TOL[dtype])


def test_noalloc_size_limit():
    dev = torch.device("cuda", 0)
    f = _bind()
    scratch = N.lib().fk_noalloc_scratch_bytes()
    assert scratch == 8 << 20
    S = N.lib().fk_decode_num_ctas(0, N.FK_DTYPE_F16, 8)
    assert S > 0
    b_max = ((scratch - 1280) // SEG_BYTES - S) // 8  # the limit stated in include/fk_decode.h (G <= 8)
    for B, ok in ((b_max, True), (b_max + 1, False)):
        lens = [40 + (i * 37) % 300 for i in range(B)]
        q, k, v, cu, s = _case(dev, lens, 32, 8, torch.float16, 128, seed=B)
        out = torch.zeros_like(q)
        rc = _call(f, q, k, v, cu, s, out)
        if ok:
            assert rc == 0, N.last_error()
            ref = fk.flash_decode_gqa_varlen(q, k, v, cu, s)
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        else:
            assert rc == 3 and "scratch" in N.last_error()
            torch.cuda.synchronize()
            assert torch.count_nonzero(out) == 0  # refused before anything was queued
    B = 4096  # far beyond the fixed scratch
    q = torch.zeros(B, 32, 128, device=dev, dtype=torch.float16)
    k = torch.zeros(B, 8, 128, device=dev, dtype=torch.float16)
    cu = torch.arange(B + 1, device=dev, dtype=torch.int32)
    assert _call(f, q, k, k, cu, None, torch.empty_like(q)) == 3
    assert _status(dev) == 0


def test_noalloc_timeout_is_reported_and_next_call_is_correct():
    # make every CTA's first pipeline wait run out (the library's test hook:
    # a stage that is never published, 50 ms bound), read the status through
    # fk_noalloc_read_status, then check that the next call is correct
    dev = torch.device("cuda", 0)
    f = _bind()
    q, k, v, cu, s = _case(dev, [20000, 9000, 4000], 32, 8, torch.float16, 128, seed=30)
    out = torch.zeros_like(q)
    L = N.lib()
    assert L.fk_debug_configure(50_000_000, 1) == 0
    try:
        assert _call(f, q, k, v, cu, s, out) == 0
        torch.cuda.synchronize()
    finally:
        assert L.fk_debug_configure(4_000_000_000, 0) == 0
    assert _status(dev, clear=1) & N.FK_STATUS_TIMEOUT
    assert _status(dev) == 0
    out = torch.full_like(q, float("nan"))
    assert _call(f, q, k, v, cu, s, out) == 0, N.last_error()
    torch.cuda.synchronize()
    assert _status(dev) == 0
    assert torch.equal(out, fk.flash_decode_gqa_varlen(q, k, v, cu, s))
