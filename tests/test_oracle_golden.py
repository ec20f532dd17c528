"""Pin the CPU oracle to the reference: golden vectors made by the reference's
own torch ``ref_attention`` and its Triton kernels (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import gqa_decode_oracle as O
from tests._golden import e4m3_to_float, load, varlen_cases


@pytest.mark.parametrize("name", varlen_cases())
def test_varlen_oracle_matches_reference_ref_attention(name):
    z = load(name)
    out = O.decode_varlen(z["q"].astype(np.float64), z["k"].astype(np.float64), z["v"].astype(np.float64),
                          z["cu_seqlens"], z.get("s_aux"))
    np.testing.assert_allclose(out, z["ref"], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("name", ["varlen_g4_nosink", "varlen_g16_nosink", "varlen_g8_d64_nosink"])
def test_varlen_oracle_matches_reference_triton_kernel_without_sinks(name):
    # K1 (triton_gqa_decode.py:35-122) run by the Triton interpreter, fp16
    # output; a 16-head group and head dim 64 included
    z = load(name)
    out = O.decode_varlen(z["q"], z["k"], z["v"], z["cu_seqlens"])
    np.testing.assert_allclose(out, z["ref_kernel"], atol=2e-3, rtol=1e-2)


def test_reference_kernels_raw_sink_diverges_from_reference_oracle():
    # The reference kernels add s_aux raw to the denominator
    # (triton_gqa_decode.py:112-115); its torch oracle adds e^(s_aux - M)
    # (tilelang_gqa_decode.py:198-203).  With s_aux ~ N(0,1) they disagree,
    # so parity is pinned to the oracle (which this library implements).
    z = load("varlen_g4_sink")
    assert np.abs(z["ref_kernel"] - z["ref"]).max() > 0.1
    z01 = load("varlen_g4_sink01")
    assert np.abs(z01["ref_kernel"] - z01["ref"]).max() > 1e-2


def test_edge_case_zero_length_rows_are_zero():
    z = load("varlen_edge_sink")
    lens = np.diff(z["cu_seqlens"])
    for b in np.nonzero(lens == 0)[0]:
        assert np.all(z["ref"][b] == 0)
    out = O.decode_varlen(z["q"], z["k"], z["v"], z["cu_seqlens"], z["s_aux"])
    np.testing.assert_allclose(out, z["ref"], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("name", ["paged_g4", "paged_g4_d64"])
def test_paged_oracle_matches_reference(name):
    z = load(name)
    out = O.decode_paged(z["q"], z["k_pool"], z["v_pool"], z["block_table"], z["seq_lens"])
    np.testing.assert_allclose(out, z["ref"], atol=2e-5, rtol=1e-5)
    # K6 (triton_paged_attn.py:19-93) under the Triton interpreter
    np.testing.assert_allclose(out, z["ref_kernel"], atol=2e-3, rtol=1e-2)


def test_dense_window_oracle_matches_reference():
    z = load("dense_g4_window")
    out = O.decode_dense(z["q"], z["k_cache"], z["v_cache"], z["cache_lens"], z["start_k_offsets"])
    np.testing.assert_allclose(out, z["ref"], atol=2e-5, rtol=1e-5)
    # K2+K3 with 4 splits (triton_gqa_decode_hf.py:18-137) under the interpreter
    np.testing.assert_allclose(out, z["ref_kernel"], atol=2e-3, rtol=1e-2)


def test_fp8_oracle_matches_reference():
    z = load("fp8_g4")
    kd = e4m3_to_float(z["k_fp8"]) * float(z["scale_k"])
    vd = e4m3_to_float(z["v_fp8"]) * float(z["scale_v"])
    # the fixture's e4m3 bytes decode to the same values torch produces
    assert np.array_equal(e4m3_to_float(z["k_fp8"]),
                          torch.from_numpy(z["k_fp8"]).view(torch.float8_e4m3fn).double().numpy())
    out = O.decode_dense(z["q"], kd, vd, z["cache_lens"])
    np.testing.assert_allclose(out, z["ref"], atol=2e-5, rtol=1e-5)
    # K4+K5 (triton_gqa_decode_hf_fp8.py:19-148): fp8 Q dequantised to fp16
    qd = (e4m3_to_float(z["q_fp8"]) * float(z["scale_q"])).astype(np.float16)
    out_q8 = O.decode_dense(qd, kd, vd, z["cache_lens"])
    np.testing.assert_allclose(out_q8, z["ref_q8"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(out_q8, z["ref_kernel"], atol=2e-3, rtol=1e-2)


def test_config1_oracle_matches_reference():
    """Benchmark config 1 (the CPU-sized case) regenerated from the seed protocol; output pinned."""
    z = load("config1_sink_fp32")
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 2049, (4,), generator=g)
    assert lens.tolist() == z["lens"].tolist() == [685, 560, 1654, 1217]
    T = int(lens.sum())
    q = torch.randn(4, 32, 128, generator=g)
    k = torch.randn(T, 8, 128, generator=g)
    v = torch.randn(T, 8, 128, generator=g)
    s = torch.randn(32, generator=g)
    np.testing.assert_allclose([q.double().sum(), k.double().sum(), v.double().sum(), s.double().sum()],
                               z["checksums"], rtol=1e-9, atol=1e-6)
    cu = np.concatenate([[0], np.cumsum(lens.numpy())])
    out = O.decode_varlen(q.numpy(), k.numpy(), v.numpy(), cu, s.numpy())
    np.testing.assert_allclose(out, z["ref"], atol=2e-5, rtol=1e-5)
