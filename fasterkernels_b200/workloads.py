"""Seeded synthetic decode workloads: the five configurations of the
benchmark plan (no dataset is involved; all inputs are random).

Lengths come from ``torch.Generator().manual_seed(seed)`` on the CPU (so they
are identical on every machine); q/k/v/s_aux are ~N(0,1), drawn on the
target device from a generator with the same seed.

  config 1  varlen fp32 (CPU oracle timing) B=4  QH=32 KVH=8  lens U[1,2048]      sinks
  config 2  varlen fp16                    B=32 QH=32 KVH=8  lens U[8192,16384]  sinks
  config 3  paged  fp16                    B=64 QH=32 KVH=8  lens U[512,8192]    no sinks, pool x1.25
  config 4  paged  e4m3 KV, fp16 Q         B=16 QH=32 KVH=8  lens 32768          sinks
  config 5  paged  e4m3 KV, fp16 Q         B=128 QH=64 KVH=8 lens logU[4096,131072] sinks
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

D = 128
PAGE = 16


@dataclass
class ConfigSpec:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    layout: str  # "varlen" | "paged"
    kv_dtype: torch.dtype
    sinks: bool
    lens_kind: str
    lens_args: tuple
    pool_factor: float = 1.25
    extra: dict = field(default_factory=dict)


CONFIGS = {
    1: ConfigSpec("config1_varlen_fp32_sinks", 4, 32, 8, "varlen", torch.float32, True, "uniform", (1, 2048)),
    2: ConfigSpec("config2_varlen_fp16_sinks", 32, 32, 8, "varlen", torch.float16, True, "uniform", (8192, 16384)),
    3: ConfigSpec("config3_paged_fp16", 64, 32, 8, "paged", torch.float16, False, "uniform", (512, 8192)),
    4: ConfigSpec("config4_paged_e4m3_sinks", 16, 32, 8, "paged", torch.float8_e4m3fn, True, "const", (32768,)),
    5: ConfigSpec("config5_paged_e4m3_sinks_longctx", 128, 64, 8, "paged", torch.float8_e4m3fn, True, "loguniform",
                  (4096, 131072)),
}


def config_lengths(cfg: int | ConfigSpec, seed: int = 0) -> list[int]:
    spec = CONFIGS[cfg] if isinstance(cfg, int) else cfg
    g = torch.Generator().manual_seed(seed)
    B = spec.batch
    if spec.lens_kind == "uniform":
        lo, hi = spec.lens_args
        return torch.randint(lo, hi + 1, (B,), generator=g).tolist()
    if spec.lens_kind == "const":
        return [spec.lens_args[0]] * B
    lo, hi = spec.lens_args
    u = torch.rand(B, generator=g, dtype=torch.float64)
    return [int(round(math.exp(float(x) * math.log(hi / lo) + math.log(lo)))) for x in u]


def kv_bytes(lens, kv_heads: int, elem_bytes: int, head_dim: int = D) -> int:
    """Algorithmic bytes of one decode step: K and V of the valid tokens."""
    return int(sum(lens)) * kv_heads * head_dim * 2 * elem_bytes


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_varlen(lens, q_heads, kv_heads, dtype, device, seed=0, sinks=True, head_dim=D):
    """q [B,QH,D], k/v [T,KVH,D], cu_seqlens [B+1] int32, s_aux [QH] fp32 or None."""
    B = len(lens)
    g = _gen(device, seed + 1)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0).to(torch.int32)
    T = int(cu[-1])
    gd = torch.float32 if dtype in (torch.float32, torch.float8_e4m3fn) else dtype
    q = torch.randn(B, q_heads, head_dim, generator=g, device=device, dtype=gd)
    k = torch.randn(T, kv_heads, head_dim, generator=g, device=device, dtype=gd)
    v = torch.randn(T, kv_heads, head_dim, generator=g, device=device, dtype=gd)
    s_aux = torch.randn(q_heads, generator=g, device=device, dtype=torch.float32) if sinks else None
    return dict(q=q, k=k, v=v, cu_seqlens=cu.to(device), s_aux=s_aux, lens=list(lens))


def varlen_to_paged(k, v, lens, pool_factor=1.25, seed=0, max_blocks=None):
    """Scatter varlen k/v [T,KVH,D] into pools [P,KVH,16,D] whose pages are a
    seeded random permutation of the pool; returns (k_pool, v_pool,
    block_table [B, max_blocks] int32 with -1 beyond each sequence)."""
    device = k.device
    B = len(lens)
    npages = [(L + PAGE - 1) // PAGE for L in lens]
    need = sum(npages)
    P = max(int(math.ceil(need * pool_factor)), 1)
    perm = torch.randperm(P, generator=torch.Generator().manual_seed(seed + 7))[:need]
    mb = max(max(npages) if npages else 1, 1) if max_blocks is None else max_blocks
    bt = torch.full((B, mb), -1, dtype=torch.int32)
    i = 0
    for b in range(B):
        bt[b, : npages[b]] = perm[i: i + npages[b]].to(torch.int32)
        i += npages[b]
    KVH, HD = k.shape[1], k.shape[2]
    k_pool = torch.zeros(P, KVH, PAGE, HD, dtype=k.dtype, device=device)
    v_pool = torch.zeros_like(k_pool)
    # token t of sequence b -> (page bt[b, t//16], slot t%16)
    starts = [0]
    for L in lens:
        starts.append(starts[-1] + L)
    phys_rows = torch.empty(starts[-1], dtype=torch.int64)
    for b in range(B):
        L = lens[b]
        if L == 0:
            continue
        t = torch.arange(L)
        phys_rows[starts[b]: starts[b] + L] = bt[b, (t // PAGE)].to(torch.int64) * PAGE + t % PAGE
    phys_rows = phys_rows.to(device)
    kf = k_pool.permute(0, 2, 1, 3).reshape(P * PAGE, KVH, HD)
    vf = v_pool.permute(0, 2, 1, 3).reshape(P * PAGE, KVH, HD)
    kf.index_copy_(0, phys_rows, k)
    vf.index_copy_(0, phys_rows, v)
    k_pool = kf.reshape(P, PAGE, KVH, HD).permute(0, 2, 1, 3).contiguous()
    v_pool = vf.reshape(P, PAGE, KVH, HD).permute(0, 2, 1, 3).contiguous()
    return k_pool, v_pool, bt.to(device)


def quantize_e4m3(x):
    """Per-tensor e4m3 quantisation with scale = amax / 448 (float32 0-dim tensor)."""
    xf = x.float()
    scale = xf.abs().max().clamp(min=1e-12) / 448.0
    return (xf / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn), scale.to(torch.float32)


def lpt_partition(lengths, n_parts: int) -> list[list[int]]:
    """Greedy longest-processing-time balance of sequences (by length, i.e. KV
    bytes) over n_parts ranks: longest first onto the least-loaded rank
    (ties -> lowest rank).  Returns the sequence indices of each rank in
    ascending order."""
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    loads = [0] * n_parts
    parts: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        r = min(range(n_parts), key=lambda j: (loads[j], j))
        parts[r].append(i)
        loads[r] += lengths[i]
    return [sorted(p) for p in parts]
