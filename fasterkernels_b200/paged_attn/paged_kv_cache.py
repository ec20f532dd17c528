"""Host-side page allocator for a paged KV cache.

Same contract as the reference's ``PagedKVCache`` and ``PAGE_SIZE``
(fskernels/paged_attn/paged_kv_cache.py:6-154): pools
[num_layers, num_pages, num_kv_heads, 16, head_dim], a device block table
[max_seqs, max_blocks_per_seq] int32 with -1 for unallocated entries, a free
list, ``allocate_sequence``/``free_sequence``/``append_kv``/
``get_block_table_tensor``/``get_seq_lens_tensor`` and the
``pages_used``/``pages_free`` counters.

Differences: the logical->physical map is mirrored on the host, so neither
``append_kv`` nor ``free_sequence`` reads the device block table back (the
reference calls ``.item()`` per appended token, paged_kv_cache.py:126);
``from_config`` honours a ``dtype`` argument (the reference hard-wires
bfloat16, :80); pools may be float8_e4m3fn.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch

PAGE_SIZE = 16


@dataclass
class PagedKVCache:
    num_layers: int
    num_pages: int
    max_seqs: int
    max_blocks_per_seq: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    device: str

    def __post_init__(self):
        shape = (self.num_layers, self.num_pages, self.num_kv_heads, PAGE_SIZE, self.head_dim)
        self.k_pool = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.block_table = torch.full((self.max_seqs, self.max_blocks_per_seq), -1, dtype=torch.int32,
                                      device=self.device)
        self._seq_lens: List[int] = [0] * self.max_seqs
        self._active: List[bool] = [False] * self.max_seqs
        self._pages: List[List[int]] = [[] for _ in range(self.max_seqs)]
        # popped from the end: lowest page indices are handed out last, as in the reference
        self._free_pages: List[int] = list(range(self.num_pages))
        # e4m3 pools store x / scale; fixed per-tensor scales (set_fp8_scales)
        self.k_scale = torch.ones((), dtype=torch.float32, device=self.device)
        self.v_scale = torch.ones((), dtype=torch.float32, device=self.device)
        self._step_ids: List[int] = []
        self._step_bt = None
        self._step_pos = None

    @classmethod
    def from_config(cls, config, num_pages: int = 4096, max_seqs: int = 16, max_blocks_per_seq: int = 512,
                    device: str = "cuda", dtype: torch.dtype = torch.bfloat16) -> "PagedKVCache":
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        return cls(num_layers=config.num_hidden_layers, num_pages=num_pages, max_seqs=max_seqs,
                   max_blocks_per_seq=max_blocks_per_seq, num_kv_heads=config.num_key_value_heads,
                   head_dim=head_dim, dtype=dtype, device=device)

    def allocate_sequence(self) -> int:
        for sid in range(self.max_seqs):
            if not self._active[sid]:
                self._active[sid] = True
                self._seq_lens[sid] = 0
                self._pages[sid] = []
                return sid
        raise RuntimeError("All sequence slots are occupied")

    def free_sequence(self, seq_id: int) -> None:
        pages = self._pages[seq_id]
        if pages:
            self.block_table[seq_id, : len(pages)] = -1
            self._free_pages.extend(pages)
        self._pages[seq_id] = []
        self._active[seq_id] = False
        self._seq_lens[seq_id] = 0

    def _alloc_page(self) -> int:
        if not self._free_pages:
            raise RuntimeError("Out of KV pages")
        return self._free_pages.pop()

    def append_kv(self, seq_id: int, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append one token's K/V ([1, KV_H, 1, D]) to a sequence of one layer."""
        pos = self._seq_lens[seq_id]
        page_idx, off = divmod(pos, PAGE_SIZE)
        pages = self._pages[seq_id]
        if page_idx == len(pages):
            if page_idx >= self.max_blocks_per_seq:
                raise RuntimeError("sequence exceeds max_blocks_per_seq")
            pp = self._alloc_page()
            pages.append(pp)
            self.block_table[seq_id, page_idx] = pp
        pp = pages[page_idx]
        self.k_pool[layer_idx, pp, :, off, :] = k[0, :, 0, :]
        self.v_pool[layer_idx, pp, :, off, :] = v[0, :, 0, :]
        self._seq_lens[seq_id] = pos + 1

    def write_prefill(self, seq_id: int, layer_idx: int, k: torch.Tensor, v: torch.Tensor, reserve: int = 0) -> None:
        """Write a prompt's K/V ([KV_H, T, D]) as tokens 0..T-1 of one layer of
        a sequence, with one indexed copy per pool (the reference appends the
        prompt token by token, benchmarks/run_hf_triton_fp8_paged.py:113-117).
        Pages are allocated on the host for max(T, reserve) tokens, so a
        caller can fix the block table for the decode steps that follow.
        The sequence length becomes T (the same T for every layer)."""
        if k.dim() != 3 or k.shape != v.shape or k.shape[0] != self.num_kv_heads or k.shape[2] != self.head_dim:
            raise ValueError("k / v must be [num_kv_heads, T, head_dim]")
        T = int(k.shape[1])
        pages = self._pages[seq_id]
        need = (max(T, int(reserve)) + PAGE_SIZE - 1) // PAGE_SIZE
        if need > self.max_blocks_per_seq:
            raise RuntimeError("sequence exceeds max_blocks_per_seq")
        if need > len(pages):
            new = [self._alloc_page() for _ in range(need - len(pages))]
            first = len(pages)
            pages.extend(new)
            self.block_table[seq_id, first:need] = torch.tensor(new, dtype=torch.int32).to(self.device)
        if T > 0:
            tok = torch.arange(T)
            phys = torch.tensor(pages, dtype=torch.long)[tok // PAGE_SIZE].to(self.device)
            slot = (tok % PAGE_SIZE).to(self.device)
            kt, vt = k.transpose(0, 1), v.transpose(0, 1)  # [T, KV_H, D]
            if self.dtype == torch.float8_e4m3fn:
                kt = (kt.float() / self.k_scale).clamp(-448.0, 448.0).to(self.dtype)
                vt = (vt.float() / self.v_scale).clamp(-448.0, 448.0).to(self.dtype)
            self.k_pool[layer_idx][phys, :, slot, :] = kt.to(self.dtype)
            self.v_pool[layer_idx][phys, :, slot, :] = vt.to(self.dtype)
        self._seq_lens[seq_id] = T

    def set_fp8_scales(self, k_scale, v_scale) -> None:
        """Per-tensor scales of an e4m3 pool (value = e4m3 x scale), e.g. amax / 448
        of calibration K/V."""
        self.k_scale.fill_(float(k_scale))
        self.v_scale.fill_(float(v_scale))

    # ---------------------------------------------------------- batched decode step
    def begin_step(self, seq_ids: List[int]):
        """Reserve the slot of one new token for each sequence in ``seq_ids``:
        pages are allocated on the host (no device read-back) and the new
        block-table entries are written with one host-to-device copy.  Returns
        (block_table [B, max_blocks], positions [B]) device tensors for
        ``append_kv_batch`` and the decode call."""
        rows, cols, vals = [], [], []
        for sid in seq_ids:
            pos = self._seq_lens[sid]
            page_idx = pos // PAGE_SIZE
            pages = self._pages[sid]
            if page_idx == len(pages):
                if page_idx >= self.max_blocks_per_seq:
                    raise RuntimeError("sequence exceeds max_blocks_per_seq")
                pp = self._alloc_page()
                pages.append(pp)
                rows.append(sid)
                cols.append(page_idx)
                vals.append(pp)
        if rows:
            upd = torch.tensor([rows, cols, vals], dtype=torch.int64).to(self.device, non_blocking=True)
            self.block_table[upd[0], upd[1]] = upd[2].to(torch.int32)
        self._step_ids = list(seq_ids)
        self._step_bt = self.get_block_table_tensor(self._step_ids)
        self._step_pos = self.get_seq_lens_tensor(self._step_ids)
        return self._step_bt, self._step_pos, self._step_pos + 1

    def append_kv_batch(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Write this step's K/V ([B, KV_H, 128] or [B, KV_H, 1, 128]) of every
        sequence of ``begin_step`` into layer ``layer_idx`` with one kernel."""
        from .paged_append import paged_kv_append
        if self._step_pos is None:
            raise RuntimeError("call begin_step() before append_kv_batch()")
        paged_kv_append(k, v, self.k_pool[layer_idx], self.v_pool[layer_idx], self._step_bt, self._step_pos,
                        scale_k=self.k_scale, scale_v=self.v_scale)

    def end_step(self) -> torch.Tensor:
        """Commit the step: every sequence of ``begin_step`` grows by one token.
        Returns the new lengths [B] (device) for the next decode call."""
        for sid in self._step_ids:
            self._seq_lens[sid] += 1
        lens = self.get_seq_lens_tensor(self._step_ids)
        self._step_ids, self._step_bt, self._step_pos = [], None, None
        return lens

    def seq_len(self, seq_id: int) -> int:
        return self._seq_lens[seq_id]

    def get_block_table_tensor(self, active_seq_ids: List[int]) -> torch.Tensor:
        idx = torch.tensor(active_seq_ids, dtype=torch.long, device=self.device)
        return self.block_table[idx]

    def get_seq_lens_tensor(self, active_seq_ids: List[int]) -> torch.Tensor:
        return torch.tensor([self._seq_lens[s] for s in active_seq_ids], dtype=torch.int32, device=self.device)

    @property
    def pages_used(self) -> int:
        return self.num_pages - len(self._free_pages)

    @property
    def pages_free(self) -> int:
        return len(self._free_pages)

    def __repr__(self) -> str:
        return (f"PagedKVCache(pages={self.num_pages}, used={self.pages_used}, "
                f"seqs={sum(self._active)}/{self.max_seqs})")
