"""Multi-GPU decode sharding (one process per GPU).

Decode attention has no cross-sequence or cross-KV-head dependency, so the
batch is partitioned with no collective on the hot path:
  * by sequence -- greedy longest-processing-time balancing of KV bytes
    (``shard_sequences``); each rank keeps the KV pages of its sequences;
  * by KV head -- when the batch is smaller than ~2x the rank count
    (``shard_kv_heads``); each rank keeps KV heads [h0, h1) and the matching
    query heads.
``gather_outputs`` assembles the per-rank outputs on every rank with one
all-gather (NCCL over NVLink on GPUs, gloo on CPU); it is off the decode hot
path and only needed when one rank wants all results.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .workloads import lpt_partition


@dataclass
class SequenceShard:
    rank: int
    world: int
    indices: list[int]      # global sequence indices owned by this rank (ascending)
    lengths: list[int]      # their lengths

    @property
    def kv_tokens(self) -> int:
        return int(sum(self.lengths))


def shard_sequences(lengths, world: int, rank: int) -> SequenceShard:
    """This rank's sequences under greedy LPT balancing of KV bytes
    (bytes are proportional to length for a fixed head count and dtype)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world {world}")
    lengths = [int(x) for x in lengths]
    idx = lpt_partition(lengths, world)[rank]
    return SequenceShard(rank, world, idx, [lengths[i] for i in idx])


def shard_kv_heads(kv_heads: int, q_heads: int, world: int, rank: int):
    """KV heads [h0, h1) and query heads [q0, q1) of this rank for a KV-head
    split (GQA groups stay whole)."""
    if kv_heads % world != 0:
        raise ValueError(f"kv_heads={kv_heads} is not divisible by world={world}")
    g = q_heads // kv_heads
    per = kv_heads // world
    h0, h1 = rank * per, (rank + 1) * per
    return (h0, h1), (h0 * g, h1 * g)


def choose_partition(batch: int, kv_heads: int, world: int) -> str:
    """'sequence' unless the batch is too small to balance (< 2 x world) and
    the KV heads divide evenly, then 'kv_head'."""
    if world > 1 and batch < 2 * world and kv_heads % world == 0:
        return "kv_head"
    return "sequence"


def gather_outputs(out_local: torch.Tensor, indices: list[int], batch: int, group=None) -> torch.Tensor:
    """All-gather per-rank outputs [B_local, Q_H, D] into the global [batch, Q_H, D]
    order given each rank's global sequence ``indices``."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dev = out_local.device
    n_local = torch.tensor([out_local.shape[0]], device=dev, dtype=torch.int64)
    sizes = [torch.zeros_like(n_local) for _ in range(world)]
    dist.all_gather(sizes, n_local, group=group)
    mx = int(max(int(s) for s in sizes))
    pad = torch.zeros((mx,) + tuple(out_local.shape[1:]), dtype=out_local.dtype, device=dev)
    pad[: out_local.shape[0]] = out_local
    idx = torch.full((mx,), -1, dtype=torch.int64, device=dev)
    idx[: len(indices)] = torch.tensor(indices, dtype=torch.int64, device=dev)
    outs = [torch.empty_like(pad) for _ in range(world)]
    idxs = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(outs, pad, group=group)
    dist.all_gather(idxs, idx, group=group)
    full = torch.empty((batch,) + tuple(out_local.shape[1:]), dtype=out_local.dtype, device=dev)
    for o, i in zip(outs, idxs):
        m = i >= 0
        full[i[m]] = o[m]
    return full
