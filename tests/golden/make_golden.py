"""Generate the golden decode-attention fixtures in tests/golden/*.npz.

Run in a container that has the reference checkout (coder0143/fasterkernels):

    FK_REFERENCE=/path/to/fasterkernels python tests/golden/make_golden.py

It imports the reference's own torch oracle ``ref_attention``
(fskernels/tilelang/tilelang_gqa_decode.py:174-207) and its FP8 helper
``quantize_to_fp8`` (fskernels/triton/triton_gqa_decode_hf_fp8.py:13-16),
and runs the reference's Triton kernels on the CPU through the Triton
interpreter (TRITON_INTERPRET=1):
  K1 flash_decode_gqa_varlen       fskernels/triton/triton_gqa_decode.py:126-155
  K2+K3 flash_decode_gqa_hf_dense_optimized  fskernels/triton/triton_gqa_decode_hf.py:146-211
  K4+K5 flash_decode_gqa_hf_fp8    fskernels/triton/triton_gqa_decode_hf_fp8.py:164-227
  K6 paged_flash_decode            fskernels/paged_attn/triton_paged_attn.py:96-125
Inputs are drawn from a seeded torch.Generator on the CPU and stored with the
outputs, so the fixtures need no reference at test time.  Sizes are kept
small (KV heads 2) so the files stay a few hundred KB each.  Names given on
the command line regenerate only those fixtures.
"""
from __future__ import annotations

import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = os.environ.get("FK_REFERENCE")
if not REF:
    raise SystemExit("set FK_REFERENCE to a checkout of the reference (coder0143/fasterkernels)")
sys.path.insert(0, REF)
OUT_DIR = os.path.dirname(os.path.abspath(__file__))

from fskernels.tilelang.tilelang_gqa_decode import ref_attention  # noqa: E402
from fskernels.triton.triton_gqa_decode import flash_decode_gqa_varlen as ref_k1  # noqa: E402
from fskernels.triton.triton_gqa_decode_hf import flash_decode_gqa_hf_dense_optimized as ref_k2  # noqa: E402
from fskernels.triton.triton_gqa_decode_hf_fp8 import flash_decode_gqa_hf_fp8 as ref_k4  # noqa: E402
from fskernels.triton.triton_gqa_decode_hf_fp8 import quantize_to_fp8, set_num_splits_fp8  # noqa: E402
from fskernels.paged_attn.triton_paged_attn import paged_flash_decode as ref_k6  # noqa: E402

D = 128


def padded_from_varlen(k, cu, B, KVH):
    lens = (cu[1:] - cu[:-1]).tolist()
    S = max(max(lens), 1)
    kp = torch.zeros(B, KVH, S, k.shape[-1], dtype=torch.float32)
    for b in range(B):
        kp[b, :, : lens[b]] = k[cu[b]: cu[b + 1]].float().transpose(0, 1)
    return kp


def oracle_ref(q, kp, vp, lens, QH, sink):
    out, _ = ref_attention(q.float(), kp, vp, torch.tensor(lens, dtype=torch.int64), QH,
                           None if sink is None else sink.float())
    return out


def varlen_case(name, seed, lens, QH, KVH, sink_scale, run_kernel, hd=D):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0).to(torch.int32)
    T = int(cu[-1])
    q = torch.randn(B, QH, hd, generator=g).half()
    k = torch.randn(T, KVH, hd, generator=g).half()
    v = torch.randn(T, KVH, hd, generator=g).half()
    sink = None if sink_scale is None else (torch.randn(QH, generator=g) * sink_scale).float()
    kp, vp = padded_from_varlen(k, cu, B, KVH), padded_from_varlen(v, cu, B, KVH)
    ref = oracle_ref(q, kp, vp, lens, QH, sink)
    rec = dict(q=q.numpy(), k=k.numpy(), v=v.numpy(), cu_seqlens=cu.numpy(), ref=ref.numpy())
    if sink is not None:
        rec["s_aux"] = sink.numpy()
    if run_kernel:
        rec["ref_kernel"] = ref_k1(q, k, v, cu, sink).float().numpy()
    np.savez_compressed(os.path.join(OUT_DIR, name + ".npz"), **rec)
    print(name, "T", T, "max|kernel-ref|",
          float(np.abs(rec["ref_kernel"] - rec["ref"]).max()) if run_kernel else "-")


def paged_case(name, seed, lens, QH, KVH, extra_pages, hd=D):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    PS = 16
    q = torch.randn(B, QH, hd, generator=g).half()
    npages = [(L + PS - 1) // PS for L in lens]
    P = sum(npages) + extra_pages
    k_pool = torch.randn(P, KVH, PS, hd, generator=g).half()
    v_pool = torch.randn(P, KVH, PS, hd, generator=g).half()
    perm = torch.randperm(P, generator=g)
    maxb = max(npages) + 1
    bt = torch.full((B, maxb), -1, dtype=torch.int32)
    i = 0
    for b in range(B):
        for p in range(npages[b]):
            bt[b, p] = int(perm[i])
            i += 1
    S = max(lens)
    kp = torch.zeros(B, KVH, S, hd)
    vp = torch.zeros(B, KVH, S, hd)
    for b in range(B):
        for p in range(npages[b]):
            n = min(PS, lens[b] - p * PS)
            kp[b, :, p * PS: p * PS + n] = k_pool[int(bt[b, p]), :, :n].float()
            vp[b, :, p * PS: p * PS + n] = v_pool[int(bt[b, p]), :, :n].float()
    ref = oracle_ref(q, kp, vp, lens, QH, None)
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    kern = ref_k6(q, k_pool, v_pool, bt, seq_lens, PS).float()
    np.savez_compressed(os.path.join(OUT_DIR, name + ".npz"), q=q.numpy(), k_pool=k_pool.numpy(),
                        v_pool=v_pool.numpy(), block_table=bt.numpy(), seq_lens=seq_lens.numpy(),
                        ref=ref.numpy(), ref_kernel=kern.numpy())
    print(name, "pages", P, "max|kernel-ref|", float((kern - ref).abs().max()))


def dense_case(name, seed, B, QH, KVH, S, lens, starts, splits):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, QH, D, generator=g).half()
    k = torch.randn(B, KVH, S, D, generator=g).half()
    v = torch.randn(B, KVH, S, D, generator=g).half()
    cache_lens = torch.tensor(lens, dtype=torch.int32)
    st = torch.tensor(starts, dtype=torch.int32)
    W = max(L - s for L, s in zip(lens, starts))
    kp = torch.zeros(B, KVH, W, D)
    vp = torch.zeros(B, KVH, W, D)
    for b in range(B):
        kp[b, :, : lens[b] - starts[b]] = k[b, :, starts[b]: lens[b]].float()
        vp[b, :, : lens[b] - starts[b]] = v[b, :, starts[b]: lens[b]].float()
    ref = oracle_ref(q, kp, vp, [L - s for L, s in zip(lens, starts)], QH, None)
    kern = ref_k2(q, k, v, cache_lens, st, num_splits=splits).float()
    np.savez_compressed(os.path.join(OUT_DIR, name + ".npz"), q=q.numpy(), k_cache=k.numpy(), v_cache=v.numpy(),
                        cache_lens=cache_lens.numpy(), start_k_offsets=st.numpy(), ref=ref.numpy(),
                        ref_kernel=kern.numpy())
    print(name, "max|kernel-ref|", float((kern - ref).abs().max()))


def fp8_case(name, seed, B, QH, KVH, S, lens, splits):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, QH, D, generator=g).half()
    k = torch.randn(B, KVH, S, D, generator=g).half()
    v = torch.randn(B, KVH, S, D, generator=g).half()
    k8, sk = quantize_to_fp8(k.float())
    v8, sv = quantize_to_fp8(v.float())
    q8, sq = quantize_to_fp8(q.float())
    cache_lens = torch.tensor(lens, dtype=torch.int32)
    kd = k8.float() * sk
    vd = v8.float() * sv
    # Oracle on fp16 Q and the dequantised KV (the configuration the new
    # library targets), and on the dequantised fp8 Q (the reference kernel's).
    ref = oracle_ref(q, kd, vd, lens, QH, None)
    ref_q8 = oracle_ref((q8.float() * sq).half(), kd, vd, lens, QH, None)
    set_num_splits_fp8(splits)
    kern = ref_k4(q8, k8, v8, cache_lens, sq, sk, sv, torch.float16).float()
    np.savez_compressed(os.path.join(OUT_DIR, name + ".npz"), q=q.numpy(), q_fp8=q8.view(torch.uint8).numpy(),
                        scale_q=np.float32(sq), k_fp8=k8.view(torch.uint8).numpy(), scale_k=np.float32(sk),
                        v_fp8=v8.view(torch.uint8).numpy(), scale_v=np.float32(sv), cache_lens=cache_lens.numpy(),
                        ref=ref.numpy(), ref_q8=ref_q8.numpy(), ref_kernel=kern.numpy())
    print(name, "max|kernel-ref_q8|", float((kern - ref_q8).abs().max()))


def config1_case():
    """Benchmark config 1 (fp32, CPU): only the output and input checksums are
    stored; the inputs are regenerated from the seed protocol (generator seed
    0: lengths, then q, k, v, s_aux)."""
    g = torch.Generator().manual_seed(0)
    B, QH, KVH = 4, 32, 8
    lens = torch.randint(1, 2049, (B,), generator=g)
    T = int(lens.sum())
    q = torch.randn(B, QH, D, generator=g)
    k = torch.randn(T, KVH, D, generator=g)
    v = torch.randn(T, KVH, D, generator=g)
    s_aux = torch.randn(QH, generator=g)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0).to(torch.int32)
    kp, vp = padded_from_varlen(k, cu, B, KVH), padded_from_varlen(v, cu, B, KVH)
    ref = oracle_ref(q, kp, vp, lens.tolist(), QH, s_aux)
    np.savez_compressed(os.path.join(OUT_DIR, "config1_sink_fp32.npz"), lens=lens.numpy(), ref=ref.numpy(),
                        checksums=np.array([q.double().sum(), k.double().sum(), v.double().sum(),
                                            s_aux.double().sum()]))
    print("config1 lens", lens.tolist())


CASES = {
    "varlen_g4_nosink": lambda: varlen_case("varlen_g4_nosink", 1, [37, 1, 200], 8, 2, None, True),
    "varlen_g4_sink": lambda: varlen_case("varlen_g4_sink", 2, [37, 1, 200], 8, 2, 1.0, True),
    "varlen_g4_sink01": lambda: varlen_case("varlen_g4_sink01", 3, [130, 64, 17], 8, 2, 0.1, True),
    "varlen_g8_sink": lambda: varlen_case("varlen_g8_sink", 4, [65, 130], 16, 2, 1.0, False),
    "varlen_edge_sink": lambda: varlen_case("varlen_edge_sink", 5, [0, 5, 16, 17, 0], 8, 2, 1.0, False),
    "paged_g4": lambda: paged_case("paged_g4", 6, [64, 33, 250, 17], 8, 2, 7),
    "dense_g4_window": lambda: dense_case("dense_g4_window", 7, 2, 8, 2, 96, [90, 50], [10, 0], 4),
    "fp8_g4": lambda: fp8_case("fp8_g4", 8, 2, 8, 2, 160, [150, 77], 2),
    "config1": config1_case,
    # shapes beyond the benchmark configs: a 16-head group (K1 pads it to BLOCK_H = 16)
    # and head dim 64 (K1 and K6 take any power of two)
    "varlen_g16_nosink": lambda: varlen_case("varlen_g16_nosink", 9, [70, 1, 150], 32, 2, None, True),
    "varlen_g8_d64_nosink": lambda: varlen_case("varlen_g8_d64_nosink", 10, [90, 3, 200], 16, 2, None, True, hd=64),
    "varlen_g4_d64_sink": lambda: varlen_case("varlen_g4_d64_sink", 11, [90, 0, 33], 8, 2, 1.0, False, hd=64),
    "paged_g4_d64": lambda: paged_case("paged_g4_d64", 12, [64, 33, 250, 17], 8, 2, 7, hd=64),
}

if __name__ == "__main__":
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name in (sys.argv[1:] or list(CASES)):
        CASES[name]()
